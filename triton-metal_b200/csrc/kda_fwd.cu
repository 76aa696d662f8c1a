// KDA (Kimi Delta Attention) chunked gated-delta-rule forward, sm_100a.
//
// No reference counterpart: triton-metal has no KDA code.  Definition (per
// head, state S in R^{Dk x Dv}, per step t):
//   S <- Diag(exp(g_t)) S;   u_t = v_t - S^T k_t;   S <- S + beta_t k_t u_t^T;
//   o_t = S^T (scale q_t)
// Chunked form over chunks of C = 64 steps (WY / UT representation of the
// product of the rank-one updates, Yang et al. 2024 "Parallelizing linear
// transformers with the delta rule"; per-channel decay as in Gated DeltaNet /
// Kimi Linear).  With G_t = cumsum of g within the chunk (G_t <= 0, per
// channel) and S the state entering the chunk:
//   A_kk[i][j] = beta_i sum_d k_i k_j exp(G_i - G_j)      (j < i)
//   A_qk[i][j] = scale sum_d q_i k_j exp(G_i - G_j)       (j <= i)
//   T = (I + A_kk)^-1,  W = T diag(beta) (K o e^G),  U = T diag(beta) V
//   V' = U - W S
//   O  = (scale Q o e^G) S + A_qk V'
//   S <- Diag(e^{G_last}) S + (K o e^{G_last - G})^T V'
//
// Kernel A (one CTA per (b, h, chunk), all chunks in parallel) computes W, U,
// Q o e^G, K o e^{G_last - G}, A_qk and e^{G_last} into a workspace.  Every
// exponent is bounded: for a 4 x 4 block of (i, j) pairs the factor
// exp(G_i - G_j) is split at r = the last row of the j block, so both
// exp(G_i - G_r) and exp(G_r - G_j) are <= 1 off the diagonal (and the
// diagonal blocks span at most 3 steps).
// Kernel B (one CTA per (b, h, 32 columns of Dv)) carries the fp32 state
// through the chunks in order on fp16 tensor cores (columns of the state are
// independent: the transition acts on the Dk side only), storing V' and each
// chunk's entering state; kernel C (parallel over chunks) forms the outputs.
#include "b2_common.cuh"

namespace b2 {
namespace kda {

constexpr int C = 64, DK = 128, DV = 128;

// Workspace block per (b, h, chunk), floats
constexpr size_t kWsW = 0;
constexpr size_t kWsU = kWsW + (size_t)C * DK;
constexpr size_t kWsQg = kWsU + (size_t)C * DV;
constexpr size_t kWsKr = kWsQg + (size_t)C * DK;
constexpr size_t kWsAq = kWsKr + (size_t)C * DK;
constexpr size_t kWsGl = kWsAq + (size_t)C * C;
constexpr size_t kWsVp = kWsGl + DK;                  // V' = U - W S (state pass -> output)
constexpr size_t kWsS = kWsVp + (size_t)C * DV;       // state entering the chunk
constexpr size_t kWsBlock = kWsS + (size_t)DK * DV;
// W, U, Kr (state pass) and Qg, A_qk, V', S_c (output pass) feed only tf32
// MMAs, whose 10-bit mantissa fp16 matches, and are O(1): they are stored as
// fp16 in the first half of their fp32-sized regions, halving the workspace
// traffic.  The state itself is carried in fp32 registers.
__device__ __forceinline__ __half* ws_h(float* blk, size_t off) { return reinterpret_cast<__half*>(blk + off); }
__device__ __forceinline__ const __half* ws_h(const float* blk, size_t off) {
  return reinterpret_cast<const __half*>(blk + off);
}
__device__ __forceinline__ uint32_t tf32(float x);
__device__ __forceinline__ uint32_t tf32h(__half x) { return tf32(__half2float(x)); }  // exact

template <typename T>
__device__ __forceinline__ float ld(const T* p) {
  if constexpr (sizeof(T) == 4) return *reinterpret_cast<const float*>(p);
  else return to_f32<T>(*p);
}
// 4 consecutive elements (16 bytes for fp32, 8 for 16-bit types) as floats
template <typename T>
__device__ __forceinline__ float4 ld4(const T* p) {
  if constexpr (sizeof(T) == 4) {
    return *reinterpret_cast<const float4*>(p);
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const T* h = reinterpret_cast<const T*>(&u);
    return make_float4(to_f32<T>(h[0]), to_f32<T>(h[1]), to_f32<T>(h[2]), to_f32<T>(h[3]));
  }
}

// ---- tf32 warp MMA (m16n8k8), fp32 accumulate -------------------------------
__device__ __forceinline__ uint32_t tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ void mma_tf32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ---------------------------------------------------------------------------
// Kernel A: intra-chunk WY/UT transform, one CTA per (b, h, chunk), 8 warps.
//  1. load K, scale*Q, g (cumsum -> G), V, beta
//  2. A_kk, A_qk on 16 x 16 blocks:
//     - off-diagonal blocks (I > J) as tf32 MMAs of bounded operands, with the
//       first row r = 16 I of block I as exponent reference:
//         K~_i = K_i e^{G_i - G_r} (i in I),  K^_j = K_j e^{G_r - G_j} (j < r)
//       (both <= 1 because G is non-increasing);
//     - diagonal blocks exactly in fp32 on CUDA cores (4 x 4 sub-blocks split
//       at their own reference rows, 4 threads per sub-block over d).
//  3. T = (I + A_kk)^-1 blockwise: diagonal 16 x 16 blocks by per-column
//     forward substitution in registers, then T_IJ = -T_II sum_M A_IM T_MJ.
//  4. W = T (beta K e^G), U = T (beta V) as tf32 MMAs.
// ---------------------------------------------------------------------------
constexpr int LD = DK + 8;   // 136: fragment reads (row g, col t) and (row t, col g) conflict-free
constexpr int LT = C + 4;    // 68
constexpr int kA2K = 0;
constexpr int kA2Q = kA2K + C * LD;   // later: beta K e^G
constexpr int kA2G = kA2Q + C * LD;
constexpr int kA2V = kA2G + C * LD;   // later: beta V
constexpr int kA2A = kA2V + C * LD;
constexpr int kA2Aq = kA2A + C * LT;
constexpr int kA2T = kA2Aq + C * LT;
constexpr int kA2Beta = kA2T + C * LT;
constexpr int kA2Floats = kA2Beta + C;
constexpr size_t kA2Smem = (size_t)kA2Floats * 4;
constexpr int kA2Threads = 512;  // 16 warps: one CTA per SM (shared memory), every phase split finer

template <typename T>
__global__ void __launch_bounds__(kA2Threads, 1)
kda_intra_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                 const float* __restrict__ g, const T* __restrict__ beta, float* __restrict__ ws, int B, int Tlen,
                 int H, float scale) {
  extern __shared__ __align__(16) float sm[];
  float* sK = sm + kA2K;
  float* sQ = sm + kA2Q;
  float* sG = sm + kA2G;
  float* sV = sm + kA2V;
  float* sA = sm + kA2A;
  float* sAq = sm + kA2Aq;
  float* sT = sm + kA2T;
  float* sBeta = sm + kA2Beta;
  const int nc = Tlen / C;
  const int chunk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;  // MMA fragment coordinates
  const int64_t row0 = ((int64_t)b * Tlen + (int64_t)chunk * C) * H + h;
  float* blk = ws + (((size_t)b * H + h) * nc + chunk) * kWsBlock;

  // ---- 1. load: g by cp.async; q, k, v as 4 consecutive d per thread, every
  // global load issued before the first shared store (latency overlapped) ----
  constexpr int kNL = C * DK / 4 / kA2Threads;  // vectors per thread per tensor
  for (int i = 0; i < kNL; ++i) {
    const int e = tid + i * kA2Threads, t = e / (DK / 4), d = 4 * (e % (DK / 4));
    cp_async16(sG + t * LD + d, g + (row0 + (int64_t)t * H) * DK + d);
  }
  cp_async_commit();
  {
    float4 kk[kNL], qq[kNL], vv[kNL];
#pragma unroll
    for (int i = 0; i < kNL; ++i) {
      const int e = tid + i * kA2Threads, t = e / (DK / 4), d = 4 * (e % (DK / 4));
      const int64_t off = (row0 + (int64_t)t * H) * DK + d;
      kk[i] = ld4(k + off);
      qq[i] = ld4(q + off);
      vv[i] = ld4(v + (row0 + (int64_t)t * H) * DV + d);
    }
#pragma unroll
    for (int i = 0; i < kNL; ++i) {
      const int e = tid + i * kA2Threads, t = e / (DK / 4), d = 4 * (e % (DK / 4));
      *reinterpret_cast<float4*>(sK + t * LD + d) = kk[i];
      *reinterpret_cast<float4*>(sQ + t * LD + d) =
          make_float4(qq[i].x * scale, qq[i].y * scale, qq[i].z * scale, qq[i].w * scale);
      *reinterpret_cast<float4*>(sV + t * LD + d) = vv[i];
    }
  }
  cp_async_wait<0>();
  if (tid < C) sBeta[tid] = ld(beta + row0 + (int64_t)tid * H);
  for (int e = tid; e < C * LT; e += kA2Threads) {
    sA[e] = 0.f;
    sAq[e] = 0.f;
  }
  __syncthreads();
  if (tid < DK) {
    float acc = 0.f;
    for (int t = 0; t < C; ++t) {
      acc += sG[t * LD + tid];
      sG[t * LD + tid] = acc;
    }
  }
  __syncthreads();

  // ---- 2a. diagonal 16 x 16 blocks, exact: 4 blocks x 10 lower 4x4 sub-blocks x 8 d-splits
  // (warps 0-9) ----
  if (tid < 320) {
    const int task = tid >> 3, split = tid & 7;
    const int D = task / 10;
    int a = 0, rem = task % 10;
    while (rem > a) {
      rem -= a + 1;
      ++a;
    }
    const int bsub = rem;  // sub-block (a, bsub), bsub <= a
    const int ib = 16 * D + 4 * a, jb = 16 * D + 4 * bsub;
    const int r = jb + 3;  // reference: last row of the j sub-block
    float akk[4][4], aqk[4][4];
#pragma unroll
    for (int x = 0; x < 4; ++x)
#pragma unroll
      for (int y = 0; y < 4; ++y) akk[x][y] = aqk[x][y] = 0.f;
    // d visits split + 8 m in an order rotated by the task's slot in the warp:
    // the 4 tasks of a warp start on rows that are multiples of 4 apart
    // (= the same bank at row stride 136), so unrotated they would read the
    // same bank; rotated, the 32 lanes cover 32 banks at every step
    const int rot = (tid >> 3) & 3;
    for (int it = 0; it < DK / 8; ++it) {
      const int d = split + 8 * ((it + rot) & (DK / 8 - 1));
      const float gr = sG[r * LD + d];
      float ki[4], qi[4], kj[4];
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        const float ei = __expf(sG[(ib + x) * LD + d] - gr);
        ki[x] = sK[(ib + x) * LD + d] * ei;
        qi[x] = sQ[(ib + x) * LD + d] * ei;
        kj[x] = sK[(jb + x) * LD + d] * __expf(gr - sG[(jb + x) * LD + d]);
      }
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) {
          akk[x][y] += ki[x] * kj[y];
          aqk[x][y] += qi[x] * kj[y];
        }
    }
#pragma unroll
    for (int x = 0; x < 4; ++x)
#pragma unroll
      for (int y = 0; y < 4; ++y) {
        akk[x][y] += __shfl_xor_sync(0xffffffffu, akk[x][y], 1);
        akk[x][y] += __shfl_xor_sync(0xffffffffu, akk[x][y], 2);
        akk[x][y] += __shfl_xor_sync(0xffffffffu, akk[x][y], 4);
        aqk[x][y] += __shfl_xor_sync(0xffffffffu, aqk[x][y], 1);
        aqk[x][y] += __shfl_xor_sync(0xffffffffu, aqk[x][y], 2);
        aqk[x][y] += __shfl_xor_sync(0xffffffffu, aqk[x][y], 4);
      }
    if (split == 0) {
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) {
          const int i = ib + x, j = jb + y;
          if (j < i) sA[i * LT + j] = akk[x][y] * sBeta[i];
          if (j <= i) sAq[i * LT + j] = aqk[x][y];
        }
    }
  }
  // ---- 2b. off-diagonal 16 x 16 blocks on tensor cores: 12 (I, n-tile) tasks,
  // run by warps 10-15 (2 each) while warps 0-9 do the diagonal blocks above
  // (disjoint outputs, shared read-only inputs) ----
  for (int task = warp - 10; warp >= 10 && task < 12; task += 6) {
    const int I = task < 2 ? 1 : (task < 6 ? 2 : 3);
    const int nt = task - (I == 1 ? 0 : (I == 2 ? 2 : 6));  // n-tile of 8 columns j in [0, 16 I)
    const int r = 16 * I;
    float ckk[4] = {0.f, 0.f, 0.f, 0.f}, cqk[4] = {0.f, 0.f, 0.f, 0.f};
    const int i0 = r + gq, i1 = r + gq + 8, j = 8 * nt + gq;
#pragma unroll 4
    for (int ks = 0; ks < DK / 8; ++ks) {
      const int d0 = 8 * ks + tq, d1 = d0 + 4;
      const float gr0 = sG[r * LD + d0], gr1 = sG[r * LD + d1];
      const float e00 = __expf(sG[i0 * LD + d0] - gr0), e10 = __expf(sG[i1 * LD + d0] - gr0);
      const float e01 = __expf(sG[i0 * LD + d1] - gr1), e11 = __expf(sG[i1 * LD + d1] - gr1);
      const uint32_t ak0 = tf32(sK[i0 * LD + d0] * e00), ak1 = tf32(sK[i1 * LD + d0] * e10);
      const uint32_t ak2 = tf32(sK[i0 * LD + d1] * e01), ak3 = tf32(sK[i1 * LD + d1] * e11);
      const uint32_t aq0 = tf32(sQ[i0 * LD + d0] * e00), aq1 = tf32(sQ[i1 * LD + d0] * e10);
      const uint32_t aq2 = tf32(sQ[i0 * LD + d1] * e01), aq3 = tf32(sQ[i1 * LD + d1] * e11);
      const uint32_t b0 = tf32(sK[j * LD + d0] * __expf(gr0 - sG[j * LD + d0]));
      const uint32_t b1 = tf32(sK[j * LD + d1] * __expf(gr1 - sG[j * LD + d1]));
      mma_tf32(ckk, ak0, ak1, ak2, ak3, b0, b1);
      mma_tf32(cqk, aq0, aq1, aq2, aq3, b0, b1);
    }
    // c0,c1: row i0, cols 8nt+2tq (+1); c2,c3: row i1
    const int jc = 8 * nt + 2 * tq;
    sA[i0 * LT + jc] = ckk[0] * sBeta[i0];
    sA[i0 * LT + jc + 1] = ckk[1] * sBeta[i0];
    sA[i1 * LT + jc] = ckk[2] * sBeta[i1];
    sA[i1 * LT + jc + 1] = ckk[3] * sBeta[i1];
    sAq[i0 * LT + jc] = cqk[0];
    sAq[i0 * LT + jc + 1] = cqk[1];
    sAq[i1 * LT + jc] = cqk[2];
    sAq[i1 * LT + jc + 1] = cqk[3];
  }
  __syncthreads();

  // ---- 3a. outputs that need raw Q / K; then beta K e^G into sQ, beta V into sV ----
  {
    const float* glr = sG + (C - 1) * LD;
    for (int e = tid; e < C * DK / 4; e += kA2Threads) {
      const int t = e / (DK / 4), d = 4 * (e % (DK / 4));
      const float bt = sBeta[t];
      const float4 gi = *reinterpret_cast<const float4*>(sG + t * LD + d);
      const float4 kk = *reinterpret_cast<const float4*>(sK + t * LD + d);
      const float4 qq = *reinterpret_cast<const float4*>(sQ + t * LD + d);
      const float4 gl = *reinterpret_cast<const float4*>(glr + d);
      float4 vv = *reinterpret_cast<const float4*>(sV + t * LD + d);
      const float4 eg = make_float4(__expf(gi.x), __expf(gi.y), __expf(gi.z), __expf(gi.w));
      {
        __half2 lo = __floats2half2_rn(qq.x * eg.x, qq.y * eg.y), hi = __floats2half2_rn(qq.z * eg.z, qq.w * eg.w);
        *reinterpret_cast<uint2*>(ws_h(blk, kWsQg) + t * DK + d) =
            make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
      }
      {
        __half2 lo = __floats2half2_rn(kk.x * __expf(gl.x - gi.x), kk.y * __expf(gl.y - gi.y));
        __half2 hi = __floats2half2_rn(kk.z * __expf(gl.z - gi.z), kk.w * __expf(gl.w - gi.w));
        *reinterpret_cast<uint2*>(ws_h(blk, kWsKr) + t * DK + d) =
            make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
      }
      *reinterpret_cast<float4*>(sQ + t * LD + d) =
          make_float4(bt * kk.x * eg.x, bt * kk.y * eg.y, bt * kk.z * eg.z, bt * kk.w * eg.w);
      vv.x *= bt;
      vv.y *= bt;
      vv.z *= bt;
      vv.w *= bt;
      *reinterpret_cast<float4*>(sV + t * LD + d) = vv;
    }
    for (int e = tid; e < C * C / 2; e += kA2Threads) {
      const int r = (2 * e) / C, c2 = (2 * e) % C;
      *reinterpret_cast<__half2*>(ws_h(blk, kWsAq) + 2 * e) =
          __floats2half2_rn(sAq[r * LT + c2], sAq[r * LT + c2 + 1]);
    }
    if (tid < DK) blk[kWsGl + tid] = __expf(glr[tid]);
  }
  // ---- 3b. diagonal blocks of T: column j of block D solved in registers ----
  if (tid < C) {
    const int D = tid >> 4, jj = tid & 15, base = 16 * D;
    float col[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float s = 0.f;
#pragma unroll
      for (int m = 0; m < 16; ++m)
        if (m > jj && m < i) s += sA[(base + i) * LT + base + m] * col[m];
      col[i] = i > jj ? -(sA[(base + i) * LT + base + jj] + s) : (i == jj ? 1.f : 0.f);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) sT[(base + i) * LT + base + jj] = col[i];
  }
  for (int e = tid; e < C * C; e += kA2Threads) {  // zero T above the diagonal blocks
    const int i = e / C, jcol = e % C;
    if ((jcol >> 4) > (i >> 4)) sT[i * LT + jcol] = 0.f;
  }
  __syncthreads();
  // ---- 3c. off-diagonal blocks of T, level by level: T_IJ = -T_II X_IJ, X_IJ = sum_{M=J}^{I-1} A_IM T_MJ ----
  for (int I = 1; I < 4; ++I) {
    float xv[3] = {0.f, 0.f, 0.f};
    const int nel = 256 * I;  // I blocks J = 0..I-1 of 16 x 16
    // X into sAq's rows of block I (A_qk is no longer needed)
    for (int e = tid; e < nel; e += kA2Threads) {
      const int J = e >> 8, ii = (e >> 4) & 15, jj = e & 15;
      float s = 0.f;
      for (int m = 16 * J; m < 16 * I; ++m) s += sA[(16 * I + ii) * LT + m] * sT[m * LT + 16 * J + jj];
      sAq[(16 * I + ii) * LT + 16 * J + jj] = s;
    }
    (void)xv;
    __syncthreads();
    for (int e = tid; e < nel; e += kA2Threads) {
      const int J = e >> 8, ii = (e >> 4) & 15, jj = e & 15;
      float s = 0.f;
      for (int m = 0; m <= ii; ++m) s += sT[(16 * I + ii) * LT + 16 * I + m] * sAq[(16 * I + m) * LT + 16 * J + jj];
      sT[(16 * I + ii) * LT + 16 * J + jj] = -s;
    }
    __syncthreads();
  }

  // ---- 4. W = T (beta K e^G), U = T (beta V): warp -> (m-tile w%4, column quarter w/4) ----
  {
    const int mt = warp & 3, nh = warp >> 2;
    const int r0 = 16 * mt, c0 = 32 * nh;
    float w[4][4], u[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) w[n][e] = u[n][e] = 0.f;
    const int ksteps = 2 * mt + 2;  // T is lower triangular
    for (int ks = 0; ks < ksteps; ++ks) {
      const int k0 = 8 * ks;
      const uint32_t a0 = tf32(sT[(r0 + gq) * LT + k0 + tq]), a1 = tf32(sT[(r0 + gq + 8) * LT + k0 + tq]);
      const uint32_t a2 = tf32(sT[(r0 + gq) * LT + k0 + tq + 4]), a3 = tf32(sT[(r0 + gq + 8) * LT + k0 + tq + 4]);
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const int col = c0 + 8 * n + gq;
        mma_tf32(w[n], a0, a1, a2, a3, tf32(sQ[(k0 + tq) * LD + col]), tf32(sQ[(k0 + tq + 4) * LD + col]));
        mma_tf32(u[n], a0, a1, a2, a3, tf32(sV[(k0 + tq) * LD + col]), tf32(sV[(k0 + tq + 4) * LD + col]));
      }
    }
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const int col = c0 + 8 * n + 2 * tq;
      const int ra = r0 + gq, rb = r0 + gq + 8;
      *reinterpret_cast<__half2*>(ws_h(blk, kWsW) + ra * DK + col) = __floats2half2_rn(w[n][0], w[n][1]);
      *reinterpret_cast<__half2*>(ws_h(blk, kWsW) + rb * DK + col) = __floats2half2_rn(w[n][2], w[n][3]);
      *reinterpret_cast<__half2*>(ws_h(blk, kWsU) + ra * DV + col) = __floats2half2_rn(u[n][0], u[n][1]);
      *reinterpret_cast<__half2*>(ws_h(blk, kWsU) + rb * DV + col) = __floats2half2_rn(u[n][2], u[n][3]);
    }
  }
}

// ---------------------------------------------------------------------------
// Kernel B: sequential state pass, one CTA per (b, h, 32 state columns).
// Per chunk (fp16 m16n8k16 MMAs with fp32 accumulate; the fp32 state lives in
// registers, its fp16 operand copy S^T in shared memory):
//   V' = U - W S          (64 x 32, K = 128)
//   S  = e^{G_last} o S + Kr^T V'   (128 x 32, K = 64; Kr^T by ldmatrix.trans)
// S and V' enter the MMAs rounded to fp16, the 10-bit mantissa tf32 gave.
// and stores V' and the state entering the chunk for kernel C.  The next
// chunk's W, Kr and U slice stream in with cp.async while this one computes.
// ---------------------------------------------------------------------------
constexpr int SV = 32;        // state columns per CTA
constexpr int kB2Threads = 128;
constexpr int LW = DK + 8;    // sW row stride (halves): A-fragment reads (row g, col t), word stride 68
constexpr int LKR = DK + 8;   // sKr row stride (halves): transposed A reads (row t, col g)
constexpr int LU = SV + 8;    // sU row stride (halves)
constexpr int LS = DK + 8;    // sSt row stride (halves): S^T, one row per state column
constexpr int LVT = C + 8;    // sVt row stride (halves): V'^T
constexpr int kB2StageBytes = (C * LW + C * LKR + C * LU) * 2;  // fp16 W, Kr, U slice
constexpr int kB2SBytes = 2 * kB2StageBytes;                    // S^T after the two stages
constexpr int kB2VtBytes = kB2SBytes + SV * LS * 2;
constexpr size_t kB2Smem = (size_t)kB2VtBytes + SV * LVT * 2;

__device__ __forceinline__ void b2_load_stage(unsigned char* st, const float* blk, int v0, int tid) {
  __half* sW = reinterpret_cast<__half*>(st);
  __half* sKr = sW + C * LW;
  __half* sU = sKr + C * LKR;
  for (int e = tid; e < C * DK / 8; e += kB2Threads) {
    const int r = e / (DK / 8), c8 = e % (DK / 8);
    cp_async16(sW + r * LW + 8 * c8, ws_h(blk, kWsW) + r * DK + 8 * c8);
    cp_async16(sKr + r * LKR + 8 * c8, ws_h(blk, kWsKr) + r * DK + 8 * c8);
  }
  for (int e = tid; e < C * SV / 8; e += kB2Threads) {
    const int r = e / (SV / 8), c8 = e % (SV / 8);
    cp_async16(sU + r * LU + 8 * c8, ws_h(blk, kWsU) + r * DV + v0 + 8 * c8);
  }
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__global__ void __launch_bounds__(kB2Threads, 1)
kda_state_kernel(float* __restrict__ ws, const float* __restrict__ s0, float* __restrict__ s_out, int B, int Tlen,
                 int H) {
  extern __shared__ __align__(16) unsigned char smb[];
  __half* sSt = reinterpret_cast<__half*>(smb + kB2SBytes);   // S^T, fp16 operand copy
  __half* sVt = reinterpret_cast<__half*>(smb + kB2VtBytes);  // V'^T, fp16 operand copy
  const int nc = Tlen / C;
  const int v0 = blockIdx.x * SV, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  float* head = ws + ((size_t)b * H + h) * nc * kWsBlock;

  b2_load_stage(smb, head, v0, tid);
  cp_async_commit();

  // state rows of this warp: m-tiles 2w, 2w+1 (dk rows 32w .. 32w+31), all 32 columns, fp32
  float acc[2][4][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = 32 * warp + 16 * mt + g + 8 * (e >> 1), col = 8 * nt + 2 * t + (e & 1);
        const float v = s0 ? s0[(((size_t)b * H + h) * DK + row) * DV + v0 + col] : 0.f;
        acc[mt][nt][e] = v;
        sSt[col * LS + row] = __float2half_rn(v);
      }

  for (int c = 0; c < nc; ++c) {
    float* blk = head + (size_t)c * kWsBlock;
    unsigned char* st = smb + (c & 1) * kB2StageBytes;
    if (c + 1 < nc) {
      b2_load_stage(smb + ((c + 1) & 1) * kB2StageBytes, blk + kWsBlock, v0, tid);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // stage c and S^T visible to all
    const __half* sW = reinterpret_cast<const __half*>(st);
    const __half* sKr = sW + C * LW;
    const __half* sU = sKr + C * LKR;

    // state entering this chunk -> workspace (read by kernel C)
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int row = 32 * warp + 16 * mt + g + 8 * (e >> 1), col = v0 + 8 * nt + 2 * t;
          *reinterpret_cast<__half2*>(ws_h(blk, kWsS) + row * DV + col) =
              __floats2half2_rn(acc[mt][nt][e], acc[mt][nt][e + 1]);
        }

    // V' = U - W S (fp16 MMAs m16n8k16, fp32 accumulate): warp w owns chunk rows 16w .. 16w+15
    {
      float p[4][4];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) p[nt][e] = 0.f;
      const int r0 = 16 * warp;
#pragma unroll 2
      for (int ks = 0; ks < DK / 16; ++ks) {
        const int k0 = 16 * ks;
        uint32_t a[4];
        a[0] = *reinterpret_cast<const uint32_t*>(sW + (r0 + g) * LW + k0 + 2 * t);
        a[1] = *reinterpret_cast<const uint32_t*>(sW + (r0 + g + 8) * LW + k0 + 2 * t);
        a[2] = *reinterpret_cast<const uint32_t*>(sW + (r0 + g) * LW + k0 + 2 * t + 8);
        a[3] = *reinterpret_cast<const uint32_t*>(sW + (r0 + g + 8) * LW + k0 + 2 * t + 8);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          uint32_t bb[2];
          bb[0] = *reinterpret_cast<const uint32_t*>(sSt + (8 * nt + g) * LS + k0 + 2 * t);
          bb[1] = *reinterpret_cast<const uint32_t*>(sSt + (8 * nt + g) * LS + k0 + 2 * t + 8);
          mma_16816<B2_F16>(p[nt], a, bb);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int row = r0 + g + 8 * (e >> 1), col = 8 * nt + 2 * t;
          const float2 u = __half22float2(*reinterpret_cast<const __half2*>(sU + row * LU + col));
          const float v0f = u.x - p[nt][e], v1f = u.y - p[nt][e + 1];
          sVt[col * LVT + row] = __float2half_rn(v0f);
          sVt[(col + 1) * LVT + row] = __float2half_rn(v1f);
          *reinterpret_cast<__half2*>(ws_h(blk, kWsVp) + row * DV + v0 + col) = __floats2half2_rn(v0f, v1f);
        }
    }
    __syncthreads();  // V'^T complete; every warp finished reading S^T

    // S = e^{G_last} o S + Kr^T V' (A = Kr^T by ldmatrix.trans, B = V'^T rows)
    {
      const float* glp = blk + kWsGl;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const float gl0 = glp[32 * warp + 16 * mt + g], gl1 = glp[32 * warp + 16 * mt + g + 8];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          acc[mt][nt][0] *= gl0;
          acc[mt][nt][1] *= gl0;
          acc[mt][nt][2] *= gl1;
          acc[mt][nt][3] *= gl1;
        }
      }
      const int mat = lane >> 3;
#pragma unroll
      for (int ks = 0; ks < C / 16; ++ks) {
        const int k0 = 16 * ks;
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          const int m0 = 32 * warp + 16 * mt;  // dk rows; A[m][k] = Kr[k][m]
          uint32_t a[4];
          ldsm_x4_trans(smem_u32(sKr + (k0 + (lane & 7) + ((mat >> 1) << 3)) * LKR + m0 + ((mat & 1) << 3)), a);
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) {
            uint32_t bb[2];
            bb[0] = *reinterpret_cast<const uint32_t*>(sVt + (8 * nt + g) * LVT + k0 + 2 * t);
            bb[1] = *reinterpret_cast<const uint32_t*>(sVt + (8 * nt + g) * LVT + k0 + 2 * t + 8);
            mma_16816<B2_F16>(acc[mt][nt], a, bb);
          }
        }
      }
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int row = 32 * warp + 16 * mt + g + 8 * (e >> 1), col = 8 * nt + 2 * t + (e & 1);
            sSt[col * LS + row] = __float2half_rn(acc[mt][nt][e]);
          }
    }
    __syncthreads();  // new S^T visible; stage c may be overwritten by the next prefetch
  }
  if (s_out) {
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = 32 * warp + 16 * mt + g + 8 * (e >> 1), col = 8 * nt + 2 * t + (e & 1);
          s_out[(((size_t)b * H + h) * DK + row) * DV + v0 + col] = acc[mt][nt][e];
        }
  }
}

// ---------------------------------------------------------------------------
// Kernel C: outputs, one CTA per (b, h, chunk), fully parallel:
//   O = (scale Q o e^G) S_c + A_qk V'     (64 x 128; fp16 MMAs on the fp16 operands)
// ---------------------------------------------------------------------------
constexpr int kCThreads = 128;
constexpr int LQ = DK + 8;   // halves; A reads (row g, col t): word stride 68 = 4 banks apart
constexpr int LAQ = C + 8;   // halves; word stride 36
constexpr int LBS = DV + 8;  // halves; B reads (row t, col g)
constexpr int kCQ = 0;
constexpr int kCA = kCQ + C * LQ;
constexpr int kCS = kCA + C * LAQ;
constexpr int kCV = kCS + DK * LBS;
constexpr int kCHalves = kCV + C * LBS;
constexpr size_t kCSmem = (size_t)kCHalves * 2;

template <typename T>
__global__ void __launch_bounds__(kCThreads, 2)
kda_output_kernel(const float* __restrict__ ws, T* __restrict__ o, int B, int Tlen, int H) {
  extern __shared__ __align__(16) __half smh[];
  __half* sQ = smh + kCQ;
  __half* sA = smh + kCA;
  __half* sS = smh + kCS;
  __half* sV = smh + kCV;
  const int nc = Tlen / C;
  const int chunk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const float* blk = ws + (((size_t)b * H + h) * nc + chunk) * kWsBlock;
  for (int e = tid; e < C * DK / 8; e += kCThreads) {
    const int r = e / (DK / 8), c8 = e % (DK / 8);
    cp_async16(sQ + r * LQ + 8 * c8, ws_h(blk, kWsQg) + r * DK + 8 * c8);
    cp_async16(sV + r * LBS + 8 * c8, ws_h(blk, kWsVp) + r * DV + 8 * c8);
  }
  for (int e = tid; e < DK * DV / 8; e += kCThreads) {
    const int r = e / (DV / 8), c8 = e % (DV / 8);
    cp_async16(sS + r * LBS + 8 * c8, ws_h(blk, kWsS) + r * DV + 8 * c8);
  }
  for (int e = tid; e < C * C / 8; e += kCThreads) {
    const int r = e / (C / 8), c8 = e % (C / 8);
    cp_async16(sA + r * LAQ + 8 * c8, ws_h(blk, kWsAq) + r * C + 8 * c8);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  // warp w: chunk rows 16w .. 16w+15, all 128 output columns (16 n-tiles)
  const int r0 = 16 * warp;
  float acc[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
  // fp16 m16n8k16 MMAs: A fragments (row-major Qg, A_qk) by 32-bit loads, B
  // fragments of the row-major [k][n] tiles (S_c, V') by ldmatrix.trans,
  // matrices (k lo, n lo), (k hi, n lo), (k lo, n hi), (k hi, n hi)
  const int mat = lane >> 3;
  const int brow = (lane & 7) + ((mat & 1) << 3), bcol = (mat >> 1) << 3;
#pragma unroll 2
  for (int ks = 0; ks < DK / 16; ++ks) {
    const int k0 = 16 * ks;
    uint32_t a[4];
    a[0] = *reinterpret_cast<const uint32_t*>(sQ + (r0 + g) * LQ + k0 + 2 * t);
    a[1] = *reinterpret_cast<const uint32_t*>(sQ + (r0 + g + 8) * LQ + k0 + 2 * t);
    a[2] = *reinterpret_cast<const uint32_t*>(sQ + (r0 + g) * LQ + k0 + 2 * t + 8);
    a[3] = *reinterpret_cast<const uint32_t*>(sQ + (r0 + g + 8) * LQ + k0 + 2 * t + 8);
#pragma unroll
    for (int np = 0; np < 8; ++np) {
      uint32_t bf[4];
      ldsm_x4_trans(smem_u32(sS + (k0 + brow) * LBS + 16 * np + bcol), bf);
      const uint32_t b0[2] = {bf[0], bf[1]}, b1[2] = {bf[2], bf[3]};
      mma_16816<B2_F16>(acc[2 * np], a, b0);
      mma_16816<B2_F16>(acc[2 * np + 1], a, b1);
    }
  }
  // A_qk is lower triangular: k-steps beyond this warp's last row contribute 0
  const int ksteps = warp + 1;
  for (int ks = 0; ks < ksteps; ++ks) {
    const int k0 = 16 * ks;
    uint32_t a[4];
    a[0] = *reinterpret_cast<const uint32_t*>(sA + (r0 + g) * LAQ + k0 + 2 * t);
    a[1] = *reinterpret_cast<const uint32_t*>(sA + (r0 + g + 8) * LAQ + k0 + 2 * t);
    a[2] = *reinterpret_cast<const uint32_t*>(sA + (r0 + g) * LAQ + k0 + 2 * t + 8);
    a[3] = *reinterpret_cast<const uint32_t*>(sA + (r0 + g + 8) * LAQ + k0 + 2 * t + 8);
#pragma unroll
    for (int np = 0; np < 8; ++np) {
      uint32_t bf[4];
      ldsm_x4_trans(smem_u32(sV + (k0 + brow) * LBS + 16 * np + bcol), bf);
      const uint32_t b0[2] = {bf[0], bf[1]}, b1[2] = {bf[2], bf[3]};
      mma_16816<B2_F16>(acc[2 * np], a, b0);
      mma_16816<B2_F16>(acc[2 * np + 1], a, b1);
    }
  }
#pragma unroll
  for (int nt = 0; nt < 16; ++nt)
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const int row = r0 + g + 8 * (e >> 1), col = 8 * nt + 2 * t;
      T* dst = o + (((int64_t)b * Tlen + (int64_t)chunk * C + row) * H + h) * DV + col;
      dst[0] = from_f32<T>(acc[nt][e]);
      dst[1] = from_f32<T>(acc[nt][e + 1]);
    }
}
}  // namespace kda
}  // namespace b2

using namespace b2;

extern "C" size_t b2_kda_workspace_size(int64_t B, int64_t T, int64_t H, int64_t Dk, int64_t Dv, int64_t chunk) {
  // 0 for every shape b2_kda_fwd rejects, and for sizes that do not fit a size_t
  if (B <= 0 || T <= 0 || H <= 0 || chunk != kda::C || T % chunk) return 0;
  if (Dk != kda::DK || Dv != kda::DV || B * H > 65535) return 0;
  const size_t per = (size_t)kda::kWsBlock * sizeof(float);
  const size_t blocks = (size_t)(B * H);
  const size_t chunks = (size_t)(T / chunk);
  if (chunks > SIZE_MAX / per / blocks) return 0;
  return blocks * chunks * per;
}

extern "C" int b2_kda_fwd(const void* q, const void* k, const void* v, const float* g, const void* beta,
                          const float* initial_state, void* o, float* final_state, void* workspace, int64_t B,
                          int64_t T, int64_t H, int64_t Dk, int64_t Dv, int64_t chunk, float scale, int dtype,
                          void* stream) {
  B2_CHECK_ARG(q && k && v && g && beta && o && workspace, B2_ERR_INVALID, "kda_fwd: null pointer");
  B2_CHECK_ARG(aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(g, 16), B2_ERR_ALIGN,
               "kda_fwd: q, k, v and g must be 16-byte aligned");
  B2_CHECK_ARG(B > 0 && T > 0 && H > 0, B2_ERR_INVALID, "kda_fwd: bad shape");
  B2_CHECK_ARG(Dk == kda::DK && Dv == kda::DV, B2_ERR_UNSUPPORTED, "kda_fwd: Dk = Dv = 128 only (got %lld, %lld)",
               (long long)Dk, (long long)Dv);
  B2_CHECK_ARG(chunk == kda::C, B2_ERR_UNSUPPORTED, "kda_fwd: chunk must be 64");
  B2_CHECK_ARG(T % chunk == 0, B2_ERR_INVALID, "kda_fwd: T=%lld must be a multiple of the chunk size",
               (long long)T);
  B2_CHECK_ARG(dtype == B2_BF16 || dtype == B2_F16 || dtype == B2_F32, B2_ERR_DTYPE, "kda_fwd: dtype %d", dtype);
  B2_CHECK_ARG(B * H <= 65535 && T / chunk <= 2147483647, B2_ERR_UNSUPPORTED, "kda_fwd: too large");
  cudaStream_t st = (cudaStream_t)stream;
  float* ws = (float*)workspace;
  const dim3 ga((unsigned)(T / chunk), (unsigned)H, (unsigned)B);
  const dim3 gb(kda::DV / kda::SV, (unsigned)H, (unsigned)B);
  set_max_smem((const void*)kda::kda_state_kernel, (int)kda::kB2Smem);
#define B2_KDA_LAUNCH(TY)                                                                                         \
  do {                                                                                                            \
    set_max_smem((const void*)kda::kda_intra_kernel<TY>, (int)kda::kA2Smem);                                     \
    set_max_smem((const void*)kda::kda_output_kernel<TY>, (int)kda::kCSmem);                                      \
    kda::kda_intra_kernel<TY><<<ga, kda::kA2Threads, kda::kA2Smem, st>>>(                                         \
        (const TY*)q, (const TY*)k, (const TY*)v, g, (const TY*)beta, ws, (int)B, (int)T, (int)H, scale);        \
    kda::kda_state_kernel<<<gb, kda::kB2Threads, kda::kB2Smem, st>>>(ws, initial_state, final_state, (int)B,     \
                                                                     (int)T, (int)H);                           \
    kda::kda_output_kernel<TY><<<ga, kda::kCThreads, kda::kCSmem, st>>>(ws, (TY*)o, (int)B, (int)T, (int)H);     \
  } while (0)
  if (dtype == B2_BF16) B2_KDA_LAUNCH(__nv_bfloat16);
  else if (dtype == B2_F16) B2_KDA_LAUNCH(__half);
  else B2_KDA_LAUNCH(float);
#undef B2_KDA_LAUNCH
  return launch_status("kda_fwd");
}

// ---------------------------------------------------------------------------
// Allocation-free variant.
//
// Some callers cannot allocate device memory at the point where they run
// KDA: code that executes while a custom allocator or memory pool must not be
// re-entered, plugin hosts that hand out only input/output buffers, or
// runtimes that forbid cudaMalloc on their hot path.  For them the workspace
// lives in a fixed file-scope device array of kNoAllocScratchBytes that every
// GPU loading this library holds until the process exits.
//
// * The first call on a device resolves the array's device address with
//   cudaGetSymbolAddress (with that device current) and caches it; make that
//   first call before any stream capture.  The cache is keyed by device
//   ordinal and assumes the runtime's primary context on that device: after
//   cudaDeviceReset, or from a different driver context, the cached address
//   is stale (call b2_kda_fwd with your own workspace there).
// * Problems whose workspace exceeds kNoAllocScratchBytes are rejected with
//   B2_ERR_INVALID (use b2_kda_fwd with a caller-provided workspace instead).
// * Every call shares the one array, which keeps the previous call's
//   contents.  Nothing in it needs clearing: each call writes every workspace
//   element it reads before reading it.  Calls whose kernels overlap on the
//   GPU (other streams, other threads) race on the array.
// ---------------------------------------------------------------------------
#include <mutex>

namespace b2 {
namespace kda {
constexpr size_t kNoAllocScratchBytes = 64ull << 20;  // 64 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static void* noalloc_scratch_ptr(int* status) {
  static std::mutex mu;
  static void* cache[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *status = B2_ERR_LAUNCH;
    set_error("kda_fwd_noalloc: no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      *status = B2_ERR_LAUNCH;
      set_error("kda_fwd_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return nullptr;
    }
    cache[dev] = p;
  }
  return cache[dev];
}
}  // namespace kda
}  // namespace b2

extern "C" int b2_kda_fwd_noalloc(const void* q, const void* k, const void* v, const float* g, const void* beta,
                                  const float* initial_state, void* o, float* final_state, int64_t B, int64_t T,
                                  int64_t H, int64_t Dk, int64_t Dv, int64_t chunk, float scale, int dtype,
                                  void* stream) {
  const size_t need = b2_kda_workspace_size(B, T, H, Dk, Dv, chunk);
  B2_CHECK_ARG(need > 0, B2_ERR_INVALID, "kda_fwd_noalloc: unsupported shape B=%lld T=%lld H=%lld chunk=%lld",
               (long long)B, (long long)T, (long long)H, (long long)chunk);
  B2_CHECK_ARG(need <= kda::kNoAllocScratchBytes, B2_ERR_INVALID,
               "kda_fwd_noalloc: workspace of %zu bytes exceeds the fixed %zu-byte device array "
               "(B*H*(T/64) <= %zu chunk-heads); call b2_kda_fwd with your own workspace",
               need, kda::kNoAllocScratchBytes, kda::kNoAllocScratchBytes / (kda::kWsBlock * sizeof(float)));
  int status = B2_OK;
  void* ws = kda::noalloc_scratch_ptr(&status);
  if (!ws) return status;
  return b2_kda_fwd(q, k, v, g, beta, initial_state, o, final_state, ws, B, T, H, Dk, Dv, chunk, scale, dtype,
                    stream);
}

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
// through the chunks in order on tf32 tensor cores (columns of the state are
// independent: the transition acts on the Dk side only), storing V' and each
// chunk's entering state; kernel C (parallel over chunks) forms the outputs.
#include "b2_common.cuh"

namespace b2 {
namespace kda {

constexpr int C = 64, DK = 128, DV = 128;
constexpr int kAThreads = 256;
constexpr int VB = 16;  // state columns per CTA in kernel B
constexpr int kBThreads = 256;
constexpr int LDA = C + 1;   // padded row stride of the 64 x 64 matrices
constexpr int LDK = DK + 1;  // padded row stride of the 64 x 128 tiles (kernel A)
constexpr int LDS = DK + 4;  // padded, 16-byte aligned row stride (kernel B)

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

template <typename T>
__device__ __forceinline__ float ld(const T* p) {
  if constexpr (sizeof(T) == 4) return *reinterpret_cast<const float*>(p);
  else return to_f32<T>(*p);
}

// smem layout of kernel A (floats)
constexpr int kAK = 0;
constexpr int kAQ = kAK + C * LDK;
constexpr int kAG = kAQ + C * LDK;
constexpr int kAV = kAG + C * LDK;
constexpr int kAAkk = kAV + C * LDK;
constexpr int kAAqk = kAAkk + C * LDA;
constexpr int kAT = kAAqk + C * LDA;
constexpr int kAKg = kAT + C * LDA;
constexpr int kABeta = kAKg + C * LDK;
constexpr int kAFloats = kABeta + C;
constexpr size_t kASmem = (size_t)kAFloats * 4;

template <typename T>
__global__ void __launch_bounds__(kAThreads, 1)
kda_intra_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                 const float* __restrict__ g, const T* __restrict__ beta, float* __restrict__ ws, int B, int Tlen,
                 int H, float scale) {
  extern __shared__ float sm[];
  float* sK = sm + kAK;
  float* sQ = sm + kAQ;
  float* sG = sm + kAG;
  float* sV = sm + kAV;
  float* sA = sm + kAAkk;
  float* sAq = sm + kAAqk;
  float* sT = sm + kAT;
  float* sKg = sm + kAKg;
  float* sBeta = sm + kABeta;
  const int nc = Tlen / C;
  const int chunk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x;
  const int64_t row0 = ((int64_t)b * Tlen + (int64_t)chunk * C) * H + h;  // (b, t0, h)
  // ---- load the chunk ----
  for (int e = tid; e < C * DK; e += kAThreads) {
    const int t = e / DK, d = e % DK;
    const int64_t off = (row0 + (int64_t)t * H) * DK + d;
    sK[t * LDK + d] = ld(k + off);
    sQ[t * LDK + d] = ld(q + off) * scale;
    sG[t * LDK + d] = g[off];
  }
  for (int e = tid; e < C * DV; e += kAThreads) {
    const int t = e / DV, d = e % DV;
    sV[t * LDK + d] = ld(v + (row0 + (int64_t)t * H) * DV + d);
  }
  if (tid < C) sBeta[tid] = ld(beta + row0 + (int64_t)tid * H);
  __syncthreads();
  // ---- cumulative decay G (per channel) ----
  if (tid < DK) {
    float acc = 0.f;
    for (int t = 0; t < C; ++t) {
      acc += sG[t * LDK + tid];
      sG[t * LDK + tid] = acc;
    }
  }
  __syncthreads();
  // ---- A_kk (j < i) and A_qk (j <= i), 4 x 4 blocks, bounded exponents ----
  if (tid < 136) {
    // map tid -> (bi, bj) with bj <= bi among 16 x 16 blocks
    int bi = 0, rem = tid;
    while (rem > bi) {
      rem -= bi + 1;
      ++bi;
    }
    const int bj = rem;
    const int r = 4 * bj + 3;  // reference row: last row of the j block
    float akk[4][4], aqk[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) akk[a][c] = aqk[a][c] = 0.f;
    for (int d = 0; d < DK; ++d) {
      const float gr = sG[r * LDK + d];
      float ki[4], qi[4], kj[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const int i = 4 * bi + a, j = 4 * bj + a;
        const float ei = __expf(sG[i * LDK + d] - gr);
        const float ej = __expf(gr - sG[j * LDK + d]);
        ki[a] = sK[i * LDK + d] * ei;
        qi[a] = sQ[i * LDK + d] * ei;
        kj[a] = sK[j * LDK + d] * ej;
      }
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          akk[a][c] += ki[a] * kj[c];
          aqk[a][c] += qi[a] * kj[c];
        }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int i = 4 * bi + a, j = 4 * bj + c;
        sA[i * LDA + j] = j < i ? akk[a][c] * sBeta[i] : 0.f;
        sAq[i * LDA + j] = j <= i ? aqk[a][c] : 0.f;
      }
  }
  // zero the upper blocks
  for (int e = tid; e < C * C; e += kAThreads) {
    const int i = e / C, j = e % C;
    if ((j >> 2) > (i >> 2)) {
      sA[i * LDA + j] = 0.f;
      sAq[i * LDA + j] = 0.f;
    }
  }
  __syncthreads();
  // ---- T = (I + A)^-1, unit lower triangular, forward substitution ----
  // thread (j, part): column j, terms m = j+1+part, +4, ... ; 4 lanes combine
  {
    const int j = tid >> 2, part = tid & 3;
    for (int i = 0; i < C; ++i) {
      float s = 0.f;
      if (j < i)
        for (int m = j + 1 + part; m < i; m += 4) s += sA[i * LDA + m] * sT[m * LDA + j];
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      if (part == 0) sT[i * LDA + j] = j < i ? -(sA[i * LDA + j] + s) : (j == i ? 1.f : 0.f);
      __syncthreads();
    }
  }
  for (int e = tid; e < C * DK; e += kAThreads) {
    const int t = e / DK, d = e % DK;
    sKg[t * LDK + d] = sK[t * LDK + d] * __expf(sG[t * LDK + d]);
  }
  __syncthreads();
  // ---- W = T diag(beta) (K o e^G), U = T diag(beta) V, and the per-row products ----
  float* blk = ws + (((size_t)b * H + h) * nc + chunk) * kWsBlock;
  {
    // thread -> (row i = tid / 4, columns d = tid % 4 + 4 c): interleaved so
    // the 4 column groups of a row fall in different banks
    const int i = tid >> 2, cg = tid & 3;
    float w[32], u[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) w[c] = u[c] = 0.f;
    for (int m = 0; m <= i; ++m) {
      const float tb = sT[i * LDA + m] * sBeta[m];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const int d = cg + 4 * c;
        w[c] += tb * sKg[m * LDK + d];
        u[c] += tb * sV[m * LDK + d];
      }
    }
    const float* gl = sG + (C - 1) * LDK;
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      const int d = cg + 4 * c;
      const float gi = sG[i * LDK + d];
      blk[kWsW + i * DK + d] = w[c];
      blk[kWsU + i * DV + d] = u[c];
      blk[kWsQg + i * DK + d] = sQ[i * LDK + d] * __expf(gi);
      blk[kWsKr + i * DK + d] = sK[i * LDK + d] * __expf(gl[d] - gi);
    }
  }
  for (int e = tid; e < C * C; e += kAThreads) blk[kWsAq + e] = sAq[(e / C) * LDA + (e % C)];
  if (tid < DK) blk[kWsGl + tid] = __expf(sG[(C - 1) * LDK + tid]);
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
// Kernel B: sequential state pass, one CTA per (b, h, 32 state columns).
// Per chunk (tf32 tensor-core MMAs, fp32 state in registers):
//   V' = U - W S          (64 x 32, K = 128)
//   S  = e^{G_last} o S + Kr^T V'   (128 x 32, K = 64)
// and stores V' and the state entering the chunk for kernel C.  The next
// chunk's W, Kr and U slice stream in with cp.async while this one computes.
// ---------------------------------------------------------------------------
constexpr int SV = 32;        // state columns per CTA
constexpr int kB2Threads = 128;
constexpr int LW = DK + 4;    // sW row stride: A-fragment reads (row g, col t) conflict-free
constexpr int LKR = DK + 8;   // sKr row stride: transposed A reads (row t, col g) conflict-free
constexpr int LB = SV + 8;    // B-operand tiles (row t, col g) conflict-free
constexpr int kB2Stage = C * LW + C * LKR + C * LB;  // floats per stage
constexpr int kB2S = 2 * kB2Stage;
constexpr int kB2Vp = kB2S + DK * LB;
constexpr int kB2Floats = kB2Vp + C * LB;
constexpr size_t kB2Smem = (size_t)kB2Floats * 4;

__device__ __forceinline__ void b2_load_stage(float* st, const float* blk, int v0, int tid) {
  float* sW = st;
  float* sKr = sW + C * LW;
  float* sU = sKr + C * LKR;
  for (int e = tid; e < C * DK / 4; e += kB2Threads) {
    const int r = e / (DK / 4), c4 = e % (DK / 4);
    cp_async16(sW + r * LW + 4 * c4, blk + kWsW + r * DK + 4 * c4);
    cp_async16(sKr + r * LKR + 4 * c4, blk + kWsKr + r * DK + 4 * c4);
  }
  for (int e = tid; e < C * SV / 4; e += kB2Threads) {
    const int r = e / (SV / 4), c4 = e % (SV / 4);
    cp_async16(sU + r * LB + 4 * c4, blk + kWsU + r * DV + v0 + 4 * c4);
  }
}

__global__ void __launch_bounds__(kB2Threads, 1)
kda_state_kernel(float* __restrict__ ws, const float* __restrict__ s0, float* __restrict__ s_out, int B, int Tlen,
                 int H) {
  extern __shared__ __align__(16) float sm[];
  float* sS = sm + kB2S;
  float* sVp = sm + kB2Vp;
  const int nc = Tlen / C;
  const int v0 = blockIdx.x * SV, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  float* head = ws + ((size_t)b * H + h) * nc * kWsBlock;

  b2_load_stage(sm, head, v0, tid);
  cp_async_commit();

  // state rows of this warp: m-tiles 2w, 2w+1 (dk rows 32w .. 32w+31), all 32 columns
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
        sS[row * LB + col] = v;
      }

  for (int c = 0; c < nc; ++c) {
    float* blk = head + (size_t)c * kWsBlock;
    float* st = sm + (c & 1) * kB2Stage;
    if (c + 1 < nc) {
      b2_load_stage(sm + ((c + 1) & 1) * kB2Stage, blk + kWsBlock, v0, tid);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // stage c and sS visible to all
    const float* sW = st;
    const float* sKr = sW + C * LW;
    const float* sU = sKr + C * LKR;

    // state entering this chunk -> workspace (read by kernel C)
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int row = 32 * warp + 16 * mt + g + 8 * (e >> 1), col = v0 + 8 * nt + 2 * t;
          *reinterpret_cast<float2*>(blk + kWsS + row * DV + col) = make_float2(acc[mt][nt][e], acc[mt][nt][e + 1]);
        }

    // V' = U - W S: warp w owns chunk rows 16w .. 16w+15
    {
      float p[4][4];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) p[nt][e] = 0.f;
      const int r0 = 16 * warp;
#pragma unroll 4
      for (int ks = 0; ks < DK / 8; ++ks) {
        const int k0 = 8 * ks;
        const uint32_t a0 = tf32(sW[(r0 + g) * LW + k0 + t]), a1 = tf32(sW[(r0 + g + 8) * LW + k0 + t]);
        const uint32_t a2 = tf32(sW[(r0 + g) * LW + k0 + t + 4]), a3 = tf32(sW[(r0 + g + 8) * LW + k0 + t + 4]);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const uint32_t b0 = tf32(sS[(k0 + t) * LB + 8 * nt + g]), b1 = tf32(sS[(k0 + t + 4) * LB + 8 * nt + g]);
          mma_tf32(p[nt], a0, a1, a2, a3, b0, b1);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int row = r0 + g + 8 * (e >> 1), col = 8 * nt + 2 * t;
          const float v0f = sU[row * LB + col] - p[nt][e], v1f = sU[row * LB + col + 1] - p[nt][e + 1];
          sVp[row * LB + col] = v0f;
          sVp[row * LB + col + 1] = v1f;
          *reinterpret_cast<float2*>(blk + kWsVp + row * DV + v0 + col) = make_float2(v0f, v1f);
        }
    }
    __syncthreads();  // V' complete; every warp finished reading sS

    // S = e^{G_last} o S + Kr^T V'
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
#pragma unroll 2
      for (int ks = 0; ks < C / 8; ++ks) {
        const int k0 = 8 * ks;
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          const int m0 = 32 * warp + 16 * mt;  // dk rows; A[m][k] = Kr[k][m]
          const uint32_t a0 = tf32(sKr[(k0 + t) * LKR + m0 + g]), a1 = tf32(sKr[(k0 + t) * LKR + m0 + g + 8]);
          const uint32_t a2 = tf32(sKr[(k0 + t + 4) * LKR + m0 + g]), a3 = tf32(sKr[(k0 + t + 4) * LKR + m0 + g + 8]);
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) {
            const uint32_t b0 = tf32(sVp[(k0 + t) * LB + 8 * nt + g]), b1 = tf32(sVp[(k0 + t + 4) * LB + 8 * nt + g]);
            mma_tf32(acc[mt][nt], a0, a1, a2, a3, b0, b1);
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
            sS[row * LB + col] = acc[mt][nt][e];
          }
    }
    __syncthreads();  // new S visible; stage c may be overwritten by the next prefetch
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
//   O = (scale Q o e^G) S_c + A_qk V'     (64 x 128; tf32 MMAs)
// ---------------------------------------------------------------------------
constexpr int kCThreads = 128;
constexpr int LQ = DK + 4;   // A reads (row g, col t)
constexpr int LAQ = C + 4;
constexpr int LBS = DV + 8;  // B reads (row t, col g)
constexpr int kCQ = 0;
constexpr int kCA = kCQ + C * LQ;
constexpr int kCS = kCA + C * LAQ;
constexpr int kCV = kCS + DK * LBS;
constexpr int kCFloats = kCV + C * LBS;
constexpr size_t kCSmem = (size_t)kCFloats * 4;

template <typename T>
__global__ void __launch_bounds__(kCThreads, 1)
kda_output_kernel(const float* __restrict__ ws, T* __restrict__ o, int B, int Tlen, int H) {
  extern __shared__ __align__(16) float sm[];
  float* sQ = sm + kCQ;
  float* sA = sm + kCA;
  float* sS = sm + kCS;
  float* sV = sm + kCV;
  const int nc = Tlen / C;
  const int chunk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const float* blk = ws + (((size_t)b * H + h) * nc + chunk) * kWsBlock;
  for (int e = tid; e < C * DK / 4; e += kCThreads) {
    const int r = e / (DK / 4), c4 = e % (DK / 4);
    cp_async16(sQ + r * LQ + 4 * c4, blk + kWsQg + r * DK + 4 * c4);
    cp_async16(sV + r * LBS + 4 * c4, blk + kWsVp + r * DV + 4 * c4);
  }
  for (int e = tid; e < DK * DV / 4; e += kCThreads) {
    const int r = e / (DV / 4), c4 = e % (DV / 4);
    cp_async16(sS + r * LBS + 4 * c4, blk + kWsS + r * DV + 4 * c4);
  }
  for (int e = tid; e < C * C / 4; e += kCThreads) {
    const int r = e / (C / 4), c4 = e % (C / 4);
    cp_async16(sA + r * LAQ + 4 * c4, blk + kWsAq + r * C + 4 * c4);
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
#pragma unroll 2
  for (int ks = 0; ks < DK / 8; ++ks) {
    const int k0 = 8 * ks;
    const uint32_t a0 = tf32(sQ[(r0 + g) * LQ + k0 + t]), a1 = tf32(sQ[(r0 + g + 8) * LQ + k0 + t]);
    const uint32_t a2 = tf32(sQ[(r0 + g) * LQ + k0 + t + 4]), a3 = tf32(sQ[(r0 + g + 8) * LQ + k0 + t + 4]);
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
      mma_tf32(acc[nt], a0, a1, a2, a3, tf32(sS[(k0 + t) * LBS + 8 * nt + g]),
               tf32(sS[(k0 + t + 4) * LBS + 8 * nt + g]));
  }
  // A_qk is lower triangular: k-steps beyond this warp's last row contribute 0
  const int ksteps = (r0 + 16) / 8;
  for (int ks = 0; ks < ksteps; ++ks) {
    const int k0 = 8 * ks;
    const uint32_t a0 = tf32(sA[(r0 + g) * LAQ + k0 + t]), a1 = tf32(sA[(r0 + g + 8) * LAQ + k0 + t]);
    const uint32_t a2 = tf32(sA[(r0 + g) * LAQ + k0 + t + 4]), a3 = tf32(sA[(r0 + g + 8) * LAQ + k0 + t + 4]);
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
      mma_tf32(acc[nt], a0, a1, a2, a3, tf32(sV[(k0 + t) * LBS + 8 * nt + g]),
               tf32(sV[(k0 + t + 4) * LBS + 8 * nt + g]));
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
  if (B <= 0 || T <= 0 || H <= 0 || chunk != kda::C || T % chunk) return 0;
  return (size_t)B * H * (T / chunk) * kda::kWsBlock * sizeof(float);
}

extern "C" int b2_kda_fwd(const void* q, const void* k, const void* v, const float* g, const void* beta,
                          const float* initial_state, void* o, float* final_state, void* workspace, int64_t B,
                          int64_t T, int64_t H, int64_t Dk, int64_t Dv, int64_t chunk, float scale, int dtype,
                          void* stream) {
  B2_CHECK_ARG(q && k && v && g && beta && o && workspace, B2_ERR_INVALID, "kda_fwd: null pointer");
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
  cudaFuncSetAttribute(kda::kda_state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kda::kB2Smem);
#define B2_KDA_LAUNCH(TY)                                                                                         \
  do {                                                                                                            \
    cudaFuncSetAttribute(kda::kda_intra_kernel<TY>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kda::kASmem); \
    cudaFuncSetAttribute(kda::kda_output_kernel<TY>, cudaFuncAttributeMaxDynamicSharedMemorySize,                 \
                         (int)kda::kCSmem);                                                                       \
    kda::kda_intra_kernel<TY><<<ga, kda::kAThreads, kda::kASmem, st>>>(                                         \
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
//   first call before any stream capture.
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

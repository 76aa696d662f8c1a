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
// Kernel B (one CTA per (b, h, 16 columns of Dv)) carries the fp32 state
// through the chunks in order.  Columns of the state are independent: the
// transition acts on the Dk side only.
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
constexpr size_t kWsBlock = kWsGl + DK;

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

// smem layout of kernel B (floats)
constexpr int kBW = 0;
constexpr int LDQ = C + 4;  // padded, 16-byte aligned row stride of A_qk (kernel B)
constexpr int kBQg = kBW + C * LDS;
constexpr int kBKr = kBQg + C * LDS;
constexpr int kBAq = kBKr + C * LDS;
constexpr int kBU = kBAq + C * LDQ;
constexpr int kBVp = kBU + C * VB;
constexpr int kBS = kBVp + C * VB;
constexpr int kBGl = kBS + DK * VB;
constexpr int kBFloats = kBGl + DK;
constexpr size_t kBSmem = (size_t)kBFloats * 4;

template <typename T>
__global__ void __launch_bounds__(kBThreads, 1)
kda_state_kernel(const float* __restrict__ ws, const float* __restrict__ s0, T* __restrict__ o,
                 float* __restrict__ s_out, int B, int Tlen, int H) {
  extern __shared__ float sm[];
  float* sW = sm + kBW;
  float* sQg = sm + kBQg;
  float* sKr = sm + kBKr;
  float* sAq = sm + kBAq;
  float* sU = sm + kBU;
  float* sVp = sm + kBVp;
  float* sS = sm + kBS;
  float* sGl = sm + kBGl;
  const int nc = Tlen / C;
  const int vb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int v0 = vb * VB;
  const int tid = threadIdx.x;
  // state slice S[:, v0:v0+VB]
  for (int e = tid; e < DK * VB; e += kBThreads) {
    const int kk = e / VB, c = e % VB;
    sS[e] = s0 ? s0[(((size_t)b * H + h) * DK + kk) * DV + v0 + c] : 0.f;
  }
  for (int chunk = 0; chunk < nc; ++chunk) {
    const float* blk = ws + (((size_t)b * H + h) * nc + chunk) * kWsBlock;
    __syncthreads();
    for (int e = tid; e < C * DK / 4; e += kBThreads) {
      const int r = e / (DK / 4), c4 = e % (DK / 4);
      reinterpret_cast<float4*>(sW + r * LDS)[c4] = reinterpret_cast<const float4*>(blk + kWsW)[e];
      reinterpret_cast<float4*>(sQg + r * LDS)[c4] = reinterpret_cast<const float4*>(blk + kWsQg)[e];
      reinterpret_cast<float4*>(sKr + r * LDS)[c4] = reinterpret_cast<const float4*>(blk + kWsKr)[e];
    }
    for (int e = tid; e < C * C / 4; e += kBThreads) {
      const int r = e / (C / 4), c4 = e % (C / 4);
      reinterpret_cast<float4*>(sAq + r * LDQ)[c4] = reinterpret_cast<const float4*>(blk + kWsAq)[e];
    }
    for (int e = tid; e < C * VB; e += kBThreads) sU[e] = blk[kWsU + (e / VB) * DV + v0 + (e % VB)];
    if (tid < DK) sGl[tid] = blk[kWsGl + tid];
    __syncthreads();
    // V' = U - W S   (64 x VB): 4 outputs per thread
    {
      const int i = tid >> 2, c0 = (tid & 3) * 4;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int kk = 0; kk < DK; ++kk) {
        const float w = sW[i * LDS + kk];
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[c] += w * sS[kk * VB + c0 + c];
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) sVp[i * VB + c0 + c] = sU[i * VB + c0 + c] - acc[c];
    }
    __syncthreads();
    // O = Qg S + Aq V'   (64 x VB)
    {
      const int i = tid >> 2, c0 = (tid & 3) * 4;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int kk = 0; kk < DK; ++kk) {
        const float qg = sQg[i * LDS + kk];
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[c] += qg * sS[kk * VB + c0 + c];
      }
      for (int j = 0; j <= i; ++j) {
        const float a = sAq[i * LDQ + j];
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[c] += a * sVp[j * VB + c0 + c];
      }
      T* orow = o + (((int64_t)b * Tlen + (int64_t)chunk * C + i) * H + h) * DV + v0 + c0;
#pragma unroll
      for (int c = 0; c < 4; ++c) orow[c] = from_f32<T>(acc[c]);
    }
    __syncthreads();
    // S <- Gl o S + Kr^T V'   (DK x VB): 8 outputs per thread
    {
      const int kk = tid >> 1, c0 = (tid & 1) * 8;
      float acc[8];
      const float gl = sGl[kk];
#pragma unroll
      for (int c = 0; c < 8; ++c) acc[c] = gl * sS[kk * VB + c0 + c];
      for (int i = 0; i < C; ++i) {
        const float kr = sKr[i * LDS + kk];
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[c] += kr * sVp[i * VB + c0 + c];
      }
      __syncthreads();  // every thread finished reading the old S
#pragma unroll
      for (int c = 0; c < 8; ++c) sS[kk * VB + c0 + c] = acc[c];
    }
  }
  __syncthreads();
  if (s_out)
    for (int e = tid; e < DK * VB; e += kBThreads) {
      const int kk = e / VB, c = e % VB;
      s_out[(((size_t)b * H + h) * DK + kk) * DV + v0 + c] = sS[e];
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
  const dim3 gb(kda::DV / kda::VB, (unsigned)H, (unsigned)B);
#define B2_KDA_LAUNCH(TY)                                                                                         \
  do {                                                                                                            \
    cudaFuncSetAttribute(kda::kda_intra_kernel<TY>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kda::kASmem); \
    cudaFuncSetAttribute(kda::kda_state_kernel<TY>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kda::kBSmem); \
    kda::kda_intra_kernel<TY><<<ga, kda::kAThreads, kda::kASmem, st>>>(                                         \
        (const TY*)q, (const TY*)k, (const TY*)v, g, (const TY*)beta, ws, (int)B, (int)T, (int)H, scale);        \
    kda::kda_state_kernel<TY><<<gb, kda::kBThreads, kda::kBSmem, st>>>(ws, initial_state, (TY*)o, final_state, \
                                                                      (int)B, (int)T, (int)H);                  \
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

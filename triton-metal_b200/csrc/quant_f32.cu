// The quantized matmuls in the reference's own dtype: fp32 activations,
// fp32 scales / zeros, fp32 output, fp32 arithmetic.
//
// Reference kernels (triton_metal/codegen/_msl_templates.py): int4_matmul
// :2716-2743 computes, per output, w = (float(q) - zeros[n][g]) * scales[n][g]
// and acc += input[m][k] * w in float; int8_matmul :2663-2677 the same with a
// per-channel scale and zero.  This file keeps exactly that arithmetic: the
// dequantised weight is formed in fp32 as (q - z) * s and every product is an
// fp32 FMA, so nothing is narrowed to 16 bits and activations of any fp32
// magnitude are representable.  It is the CUDA-core path the entry points
// take for dtype B2_F32; the 16-bit activations run the tensor-core kernels.
//
// Layouts: 0 = GPTQ int32 [K/8, N] (nibble j = k % 8) with scales / zeros
// [K/G, N]; 1 = the reference's uint8 [N, K/2] (low nibble = even k) with
// scales / zeros [N, K/G]; 2 = int8 [N, K] with per-channel scales / zeros [N].
//
// One CTA covers 64 output columns x MB rows of M; its 4 x 64 threads split
// the K groups of a column 4 ways (groups ks, ks + 4, ...) and reduce through
// shared memory.  A warp reads 32 consecutive columns of a GPTQ row (128 B,
// coalesced); x is read as 16-byte vectors that every lane of a warp shares.
#include "b2_common.cuh"

namespace b2 {
namespace qf32 {

constexpr int kCols = 64, kSplit = 4, kThreads = kCols * kSplit;

template <int LAYOUT>
__device__ __forceinline__ uint32_t load_word(const void* w, int N, int K, int n, int kw) {
  if constexpr (LAYOUT == 0) return reinterpret_cast<const uint32_t*>(w)[(size_t)(kw >> 3) * N + n];
  else if constexpr (LAYOUT == 1)
    return reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint8_t*>(w) + (size_t)n * (K / 2))[kw >> 3];
  else return reinterpret_cast<const uint32_t*>(reinterpret_cast<const int8_t*>(w) + (size_t)n * K)[kw >> 2];
}

template <int LAYOUT, int MB>
__global__ void __launch_bounds__(kThreads)
quant_f32_kernel(const float* __restrict__ x, const void* __restrict__ w, float* __restrict__ out,
                 const float* __restrict__ s, const float* __restrict__ z, int M, int N, int K, int G) {
  __shared__ float red[kSplit - 1][MB][kCols];
  constexpr int KPW = LAYOUT == 2 ? 4 : 8;  // k per 32-bit weight word
  const int col = threadIdx.x % kCols, ks = threadIdx.x / kCols;
  const int n = blockIdx.x * kCols + col, m0 = blockIdx.y * MB;
  const int gk = LAYOUT == 2 ? 128 : G;  // k per work unit (int8: a fixed slice, same channel scale)
  const int nunits = (K + gk - 1) / gk;
  float acc[MB];
#pragma unroll
  for (int m = 0; m < MB; ++m) acc[m] = 0.f;
  if (n < N) {
    for (int u = ks; u < nunits; u += kSplit) {
      float sc, zc;
      if constexpr (LAYOUT == 0) {
        sc = s[(size_t)u * N + n];
        zc = z ? z[(size_t)u * N + n] : 8.f;
      } else if constexpr (LAYOUT == 1) {
        sc = s[(size_t)n * (K / G) + u];
        zc = z ? z[(size_t)n * (K / G) + u] : 8.f;
      } else {
        sc = s[n];
        zc = z ? z[n] : 0.f;
      }
      const int k1 = min(K, (u + 1) * gk);
      for (int kw = u * gk; kw < k1; kw += KPW) {
        const uint32_t word = load_word<LAYOUT>(w, N, K, n, kw);
        float wv[KPW];
#pragma unroll
        for (int j = 0; j < KPW; ++j) {
          const float q = LAYOUT == 2 ? (float)(int)(int8_t)(word >> (8 * j)) : (float)((word >> (4 * j)) & 0xFu);
          wv[j] = (q - zc) * sc;  // the reference's float dequant, rounded once like it
        }
#pragma unroll
        for (int m = 0; m < MB; ++m) {
          if (m0 + m < M) {
            const float* xr = x + (size_t)(m0 + m) * K + kw;
#pragma unroll
            for (int j4 = 0; j4 < KPW; j4 += 4) {
              const float4 xv = __ldg(reinterpret_cast<const float4*>(xr + j4));
              acc[m] = fmaf(xv.x, wv[j4], acc[m]);
              acc[m] = fmaf(xv.y, wv[j4 + 1], acc[m]);
              acc[m] = fmaf(xv.z, wv[j4 + 2], acc[m]);
              acc[m] = fmaf(xv.w, wv[j4 + 3], acc[m]);
            }
          }
        }
      }
    }
  }
  if (ks > 0) {
#pragma unroll
    for (int m = 0; m < MB; ++m) red[ks - 1][m][col] = acc[m];
  }
  __syncthreads();
  if (ks == 0 && n < N) {
#pragma unroll
    for (int m = 0; m < MB; ++m) {
      if (m0 + m < M) {
        float v = acc[m];
#pragma unroll
        for (int r = 0; r < kSplit - 1; ++r) v += red[r][m][col];
        out[(size_t)(m0 + m) * N + n] = v;
      }
    }
  }
}

template <int LAYOUT>
int launch(const void* x, const void* w, void* out, const void* s, const void* z, int64_t M, int64_t N, int64_t K,
           int64_t G, cudaStream_t st) {
  const unsigned gx = (unsigned)((N + kCols - 1) / kCols);
  const auto X = (const float*)x;
  const auto O = (float*)out;
  const auto S = (const float*)s;
  const auto Z = (const float*)z;
#define B2_QF32(MB)                                                                                   \
  do {                                                                                                \
    const dim3 grid(gx, (unsigned)((M + (MB)-1) / (MB)));                                             \
    quant_f32_kernel<LAYOUT, MB><<<grid, kThreads, 0, st>>>(X, w, O, S, Z, (int)M, (int)N, (int)K, (int)G); \
  } while (0)
  if (M <= 1) B2_QF32(1);
  else if (M <= 2) B2_QF32(2);
  else if (M <= 4) B2_QF32(4);
  else if (M <= 8) B2_QF32(8);
  else B2_QF32(16);
#undef B2_QF32
  return launch_status("quant_f32");
}

}  // namespace qf32

// fp32 entry used by b2_int4_matmul (layout 0), b2_int4_matmul_ref (1) and
// b2_int8_matmul (2) for dtype B2_F32; shapes already validated by the caller.
int b2_detail_quant_f32(int layout, const void* x, const void* w, void* out, const void* s, const void* z,
                        int64_t M, int64_t N, int64_t K, int64_t G, cudaStream_t st) {
  B2_CHECK_ARG(aligned(x, 16) && aligned(w, 4), B2_ERR_ALIGN, "quantized matmul (fp32): x must be 16-byte aligned");
  B2_CHECK_ARG(K % 8 == 0, B2_ERR_INVALID, "quantized matmul (fp32): K=%lld must be a multiple of 8", (long long)K);
  B2_CHECK_ARG(layout == 2 || (G % 8 == 0 && K % G == 0), B2_ERR_INVALID,
               "quantized matmul (fp32): group_size=%lld must be a multiple of 8 dividing K", (long long)G);
  if (layout == 0) return qf32::launch<0>(x, w, out, s, z, M, N, K, G, st);
  if (layout == 1) return qf32::launch<1>(x, w, out, s, z, M, N, K, G, st);
  return qf32::launch<2>(x, w, out, s, z, M, N, K, G, st);
}

}  // namespace b2

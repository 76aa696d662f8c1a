// W4A16 group-wise weight-only matmul: decode GEMV (M <= 16), the exact
// dequant export, the reference->GPTQ repack, and a generic per-output
// kernel for shapes outside the fast paths' constraints.
//
// Math (reference int4_matmul, triton_metal/codegen/_msl_templates.py:2716-2743):
//   out[m,n] = sum_k x[m,k] * (q[k,n] - z[g,n]) * s[g,n],  g = k / G.
//
// Decode GEMV design (HBM-bound, 0.5 byte of weight per MAC):
//   * CTA = 8 warps, tile of 32 output columns; the K groups are split
//     across the 8 warps and the partials reduced in shared memory.
//   * Lane (g = lane/4, t = lane%4) loads one 128-bit word of the packed
//     weight: 4 adjacent columns x 8 k of GPTQ row (4*step + t).  A warp
//     load therefore covers 4 rows x 128 contiguous bytes.
//   * Nibbles become exact small integers (q - 8) in the activation dtype
//     with the magic-exponent trick (q | 0x6400 is 1024 + q in fp16,
//     q | 0x4300 is 128 + q in bf16; one LOP3 + one packed SUB per pair).
//   * Products run on mma.sync m16n8k16 with the WEIGHTS as the A operand
//     (16 columns x 16 k) and x^T as B (16 k x 8 rows of M), so M <= 8
//     needs one n-tile and M <= 16 two.  k inside an MMA is permuted
//     consistently on both operands: lane t's slots {2t,2t+1} hold nibbles
//     (j, j+4) of its own word, and x is permuted to match with PRMT.
//   * Each group's MMA sum is exact-integer-weighted and is scaled in fp32
//     by the group scale afterwards: acc += s * (C_g - (z - 8) * sum_g(x)).
#include "b2_common.cuh"

namespace b2 {

constexpr int kGemvWarps = 8;
constexpr int kGemvCols = 32;

template <int DT>
struct Magic;
template <>
struct Magic<B2_F16> {
  static constexpr uint32_t base = 0x64006400u;   // (1024, 1024)
  static constexpr uint32_t base8 = 0x64086408u;  // (1032, 1032)
};
template <>
struct Magic<B2_BF16> {
  static constexpr uint32_t base = 0x43004300u;   // (128, 128)
  static constexpr uint32_t base8 = 0x43084308u;  // (136, 136)
};

template <int DT>
__device__ __forceinline__ float2 unpack2(uint32_t v) {
  using T2 = typename dtype_of<DT>::T2;
  T2 h = *reinterpret_cast<T2*>(&v);
  if constexpr (DT == B2_F16) return __half22float2(h);
  else return __bfloat1622float2(h);
}

// One 128-bit word of x (8 consecutive k of one row) -> the B fragment
// pairs (k, k+4) used by the permuted-k MMA.
__device__ __forceinline__ void x_pairs(const uint4& xv, uint32_t (&p)[4]) {
  p[0] = prmt(xv.x, xv.z, 0x5410);
  p[1] = prmt(xv.x, xv.z, 0x7632);
  p[2] = prmt(xv.y, xv.w, 0x5410);
  p[3] = prmt(xv.y, xv.w, 0x7632);
}

// SPG = 128-bit steps per group (G = 32 * SPG); NT = n-tiles of 8 rows of M.
template <int DT, int NT, int SPG, bool ZEROS>
__global__ void __launch_bounds__(kGemvWarps * 32)
w4_gemv_kernel(const uint16_t* __restrict__ x, const uint32_t* __restrict__ qw,
               uint16_t* __restrict__ out, const uint16_t* __restrict__ scales,
               const uint16_t* __restrict__ zeros, int M, int N, int K) {
  using T = typename dtype_of<DT>::T;
  __shared__ float red[kGemvWarps][NT * 8 * kGemvCols];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int col0 = blockIdx.x * kGemvCols;
  const int colbase = col0 + 4 * g;
  const bool cvalid = colbase < N;
  const int ngroups = K / (32 * SPG);
  const int per_warp = (ngroups + kGemvWarps - 1) / kGemvWarps;
  const int g_begin = warp * per_warp;
  const int g_end = min(ngroups, g_begin + per_warp);

  float acc[2][NT][4];
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int b = 0; b < NT; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;

  const uint32_t* wp = qw + colbase;
  uint4 wcur[SPG], wnext[SPG];
  if (g_begin < g_end) {
#pragma unroll
    for (int s = 0; s < SPG; ++s) {
      int row = g_begin * 4 * SPG + 4 * s + t;
      wcur[s] = cvalid ? ld_stream_u4(wp + (size_t)row * N) : make_uint4(0, 0, 0, 0);
    }
  }

  for (int grp = g_begin; grp < g_end; ++grp) {
    // prefetch the next group's weights while this one is computed
    if (grp + 1 < g_end) {
#pragma unroll
      for (int s = 0; s < SPG; ++s) {
        int row = (grp + 1) * 4 * SPG + 4 * s + t;
        wnext[s] = cvalid ? ld_stream_u4(wp + (size_t)row * N) : make_uint4(0, 0, 0, 0);
      }
    }
    float sc[4], zc[4];
    {
      uint2 sv = cvalid ? __ldg(reinterpret_cast<const uint2*>(scales + (size_t)grp * N + colbase))
                        : make_uint2(0, 0);
      float2 a = unpack2<DT>(sv.x), b = unpack2<DT>(sv.y);
      sc[0] = a.x; sc[1] = a.y; sc[2] = b.x; sc[3] = b.y;
      if constexpr (ZEROS) {
        uint2 zv = cvalid ? __ldg(reinterpret_cast<const uint2*>(zeros + (size_t)grp * N + colbase))
                          : make_uint2(0, 0);
        float2 c = unpack2<DT>(zv.x), d = unpack2<DT>(zv.y);
        zc[0] = c.x - 8.f; zc[1] = c.y - 8.f; zc[2] = d.x - 8.f; zc[3] = d.y - 8.f;
      }
    }
    float cg[2][NT][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int b = 0; b < NT; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) cg[a][b][c] = 0.f;
    float xs[NT];
#pragma unroll
    for (int b = 0; b < NT; ++b) xs[b] = 0.f;

#pragma unroll
    for (int s = 0; s < SPG; ++s) {
      const int row = grp * 4 * SPG + 4 * s + t;
      uint32_t bp[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int m = g + 8 * nt;
        uint4 xv = make_uint4(0, 0, 0, 0);
        if (m < M) xv = __ldg(reinterpret_cast<const uint4*>(x + (size_t)m * K + 8 * row));
        x_pairs(xv, bp[nt]);
        if constexpr (ZEROS) {
          float2 a = unpack2<DT>(xv.x), b = unpack2<DT>(xv.y), c = unpack2<DT>(xv.z), d = unpack2<DT>(xv.w);
          xs[nt] += (a.x + a.y) + (b.x + b.y) + (c.x + c.y) + (d.x + d.y);
        }
      }
      const uint32_t wv[4] = {wcur[s].x, wcur[s].y, wcur[s].z, wcur[s].w};
      uint32_t dq[4][4];
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          dq[c][j] = sub2<DT>(and_or(wv[c] >> (4 * j), 0x000F000Fu, Magic<DT>::base), Magic<DT>::base8);
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const uint32_t a0[4] = {dq[2 * mt][0], dq[2 * mt + 1][0], dq[2 * mt][1], dq[2 * mt + 1][1]};
        const uint32_t a1[4] = {dq[2 * mt][2], dq[2 * mt + 1][2], dq[2 * mt][3], dq[2 * mt + 1][3]};
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint32_t b0[2] = {bp[nt][0], bp[nt][1]};
          const uint32_t b1[2] = {bp[nt][2], bp[nt][3]};
          mma_16816<DT>(cg[mt][nt], a0, b0);
          mma_16816<DT>(cg[mt][nt], a1, b1);
        }
      }
    }
    // fold the group into the fp32 accumulator with its scale (and zero)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float x0 = 0.f, x1 = 0.f;
      if constexpr (ZEROS) {
        float tot = xs[nt];
        tot += __shfl_xor_sync(0xffffffffu, tot, 1);
        tot += __shfl_xor_sync(0xffffffffu, tot, 2);
        // tot = sum_g x[8nt + g]; C columns of this lane are m = 8nt+2t, +1
        x0 = __shfl_sync(0xffffffffu, tot, (2 * t) << 2);
        x1 = __shfl_sync(0xffffffffu, tot, (2 * t + 1) << 2);
      }
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const float s0 = sc[2 * mt], s1 = sc[2 * mt + 1];
        if constexpr (ZEROS) {
          const float z0 = zc[2 * mt], z1 = zc[2 * mt + 1];
          acc[mt][nt][0] += s0 * (cg[mt][nt][0] - z0 * x0);
          acc[mt][nt][1] += s0 * (cg[mt][nt][1] - z0 * x1);
          acc[mt][nt][2] += s1 * (cg[mt][nt][2] - z1 * x0);
          acc[mt][nt][3] += s1 * (cg[mt][nt][3] - z1 * x1);
        } else {
          acc[mt][nt][0] += s0 * cg[mt][nt][0];
          acc[mt][nt][1] += s0 * cg[mt][nt][1];
          acc[mt][nt][2] += s1 * cg[mt][nt][2];
          acc[mt][nt][3] += s1 * cg[mt][nt][3];
        }
      }
    }
#pragma unroll
    for (int s = 0; s < SPG; ++s) wcur[s] = wnext[s];
  }

  // per-warp partials -> shared memory -> sum over warps
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const int m = nt * 8 + 2 * t;
      const int c = 4 * g + 2 * mt;
      red[warp][m * kGemvCols + c] = acc[mt][nt][0];
      red[warp][(m + 1) * kGemvCols + c] = acc[mt][nt][1];
      red[warp][m * kGemvCols + c + 1] = acc[mt][nt][2];
      red[warp][(m + 1) * kGemvCols + c + 1] = acc[mt][nt][3];
    }
  __syncthreads();
  for (int i = threadIdx.x; i < NT * 8 * kGemvCols; i += blockDim.x) {
    const int m = i / kGemvCols, c = i % kGemvCols;
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < kGemvWarps; ++w) sum += red[w][i];
    if (m < M && col0 + c < N) {
      T r = from_f32<T>(sum);
      out[(size_t)m * N + col0 + c] = *reinterpret_cast<uint16_t*>(&r);
    }
  }
}

// Generic kernel: one thread per output, any M/N/K/G, GPTQ layout.  Used for
// shapes outside the fast paths (tiny K, G not a multiple of 32, odd N).
template <int DT>
__global__ void w4_generic_kernel(const uint16_t* __restrict__ x, const uint32_t* __restrict__ qw,
                                  uint16_t* __restrict__ out, const uint16_t* __restrict__ scales,
                                  const uint16_t* __restrict__ zeros, int M, int N, int K, int G) {
  using T = typename dtype_of<DT>::T;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)M * N) return;
  const int m = idx / N, n = idx % N;
  float acc = 0.f, gacc = 0.f, gx = 0.f;
  for (int k = 0; k < K; ++k) {
    const uint32_t word = qw[(size_t)(k >> 3) * N + n];
    const float q = (float)((word >> (4 * (k & 7))) & 0xF);
    const float xv = to_f32<T>(*reinterpret_cast<const T*>(x + (size_t)m * K + k));
    gacc += xv * (q - 8.f);
    gx += xv;
    if ((k + 1) % G == 0 || k + 1 == K) {
      const int grp = k / G;
      const float s = to_f32<T>(*reinterpret_cast<const T*>(scales + (size_t)grp * N + n));
      const float z = zeros ? to_f32<T>(*reinterpret_cast<const T*>(zeros + (size_t)grp * N + n)) - 8.f : 0.f;
      acc += s * (gacc - z * gx);
      gacc = 0.f;
      gx = 0.f;
    }
  }
  T r = from_f32<T>(acc);
  out[idx] = *reinterpret_cast<uint16_t*>(&r);
}

// Exact dequant: W[k,n] = (q - z) * float(s) in fp32.
template <int DT>
__global__ void w4_dequant_kernel(const uint32_t* __restrict__ qw, const uint16_t* __restrict__ scales,
                                  const uint16_t* __restrict__ zeros, float* __restrict__ out,
                                  int N, int K, int G) {
  using T = typename dtype_of<DT>::T;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)K * N) return;
  const int k = idx / N, n = idx % N;
  const uint32_t word = qw[(size_t)(k >> 3) * N + n];
  const float q = (float)((word >> (4 * (k & 7))) & 0xF);
  const int grp = k / G;
  const float s = to_f32<T>(*reinterpret_cast<const T*>(scales + (size_t)grp * N + n));
  const float z = zeros ? to_f32<T>(*reinterpret_cast<const T*>(zeros + (size_t)grp * N + n)) : 8.f;
  out[idx] = (q - z) * s;
}

// uint8 [N, K/2] (low nibble = even k) -> int32 [K/8, N]
__global__ void w4_repack_kernel(const uint8_t* __restrict__ ref, uint32_t* __restrict__ gptq, int N, int K) {
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)(K / 8) * N) return;
  const int r = idx / N, n = idx % N;
  const uint32_t lo = *reinterpret_cast<const uint32_t*>(ref + (size_t)n * (K / 2) + 4 * r);
  // bytes b0..b3 hold k = 8r+0..7 as (lo nibble even, hi nibble odd): the
  // nibble order in a little-endian word already is k order.
  gptq[idx] = lo;
}

template <int DT, int NT, int SPG>
static void launch_gemv(const void* x, const void* w, void* out, const void* s, const void* z,
                        int M, int N, int K, cudaStream_t st) {
  dim3 grid((N + kGemvCols - 1) / kGemvCols);
  if (z)
    w4_gemv_kernel<DT, NT, SPG, true><<<grid, kGemvWarps * 32, 0, st>>>(
        (const uint16_t*)x, (const uint32_t*)w, (uint16_t*)out, (const uint16_t*)s, (const uint16_t*)z, M, N, K);
  else
    w4_gemv_kernel<DT, NT, SPG, false><<<grid, kGemvWarps * 32, 0, st>>>(
        (const uint16_t*)x, (const uint32_t*)w, (uint16_t*)out, (const uint16_t*)s, nullptr, M, N, K);
}

template <int DT>
static int gemv_dispatch(const void* x, const void* w, void* out, const void* s, const void* z,
                         int M, int N, int K, int G, cudaStream_t st) {
  const int spg = G / 32;
#define B2_SPG_CASE(S)                                      \
  case S:                                                   \
    if (M <= 8) launch_gemv<DT, 1, S>(x, w, out, s, z, M, N, K, st); \
    else launch_gemv<DT, 2, S>(x, w, out, s, z, M, N, K, st);        \
    break;
  switch (spg) {
    B2_SPG_CASE(1)
    B2_SPG_CASE(2)
    B2_SPG_CASE(4)
    B2_SPG_CASE(8)
    default: return B2_ERR_UNSUPPORTED;
  }
#undef B2_SPG_CASE
  return launch_status("w4_gemv");
}

// Returns true when the decode GEMV's layout constraints hold.
static bool gemv_ok(const void* x, const void* w, const void* s, const void* z,
                    int64_t M, int64_t N, int64_t K, int64_t G) {
  return M >= 1 && M <= 16 && N % 4 == 0 && K % G == 0 && G % 32 == 0 && G / 32 <= 8 &&
         (G / 32 & (G / 32 - 1)) == 0 && aligned(x, 16) && aligned(w, 16) && aligned(s, 8) &&
         (!z || aligned(z, 8));
}

}  // namespace b2

using namespace b2;

// Implemented in wxa16_gemm_sm100.cu: tcgen05 prefill GEMM for M > 16.
int b2_detail_w4_gemm(const void* x, const void* w, void* out, const void* s, const void* z,
                      int64_t M, int64_t N, int64_t K, int64_t G, int dtype, cudaStream_t st);

extern "C" int b2_int4_matmul(const void* input, const void* weight, void* output,
                              const void* scales, const void* zeros,
                              int64_t M, int64_t N, int64_t K, int64_t group_size,
                              int dtype, void* stream) {
  B2_CHECK_ARG(input && weight && output && scales, B2_ERR_INVALID, "int4_matmul: null pointer");
  B2_CHECK_ARG(M >= 0 && N > 0 && K > 0, B2_ERR_INVALID, "int4_matmul: bad shape M=%lld N=%lld K=%lld",
               (long long)M, (long long)N, (long long)K);
  B2_CHECK_ARG(K % 8 == 0, B2_ERR_INVALID, "int4_matmul: K=%lld must be a multiple of 8 (GPTQ packing)",
               (long long)K);
  B2_CHECK_ARG(group_size > 0 && K % group_size == 0, B2_ERR_INVALID,
               "int4_matmul: group_size=%lld must divide K=%lld", (long long)group_size, (long long)K);
  B2_CHECK_ARG(dtype == B2_F16 || dtype == B2_BF16, B2_ERR_DTYPE, "int4_matmul: dtype %d unsupported", dtype);
  B2_CHECK_ARG(M * N < (1ll << 31) && K * N / 8 < (1ll << 31), B2_ERR_UNSUPPORTED, "int4_matmul: too large");
  if (M == 0) return B2_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (gemv_ok(input, weight, scales, zeros, M, N, K, group_size)) {
    return dtype == B2_F16 ? gemv_dispatch<B2_F16>(input, weight, output, scales, zeros, M, N, K, group_size, st)
                           : gemv_dispatch<B2_BF16>(input, weight, output, scales, zeros, M, N, K, group_size, st);
  }
  if (M > 16) {
    int r = b2_detail_w4_gemm(input, weight, output, scales, zeros, M, N, K, group_size, dtype, st);
    if (r != B2_ERR_UNSUPPORTED) return r;
  }
  const long total = M * N;
  const int blocks = (int)((total + 255) / 256);
  if (dtype == B2_F16)
    w4_generic_kernel<B2_F16><<<blocks, 256, 0, st>>>((const uint16_t*)input, (const uint32_t*)weight,
                                                      (uint16_t*)output, (const uint16_t*)scales,
                                                      (const uint16_t*)zeros, M, N, K, group_size);
  else
    w4_generic_kernel<B2_BF16><<<blocks, 256, 0, st>>>((const uint16_t*)input, (const uint32_t*)weight,
                                                       (uint16_t*)output, (const uint16_t*)scales,
                                                       (const uint16_t*)zeros, M, N, K, group_size);
  return launch_status("w4_generic");
}

extern "C" int b2_int4_dequant(const void* weight, const void* scales, const void* zeros, float* out,
                               int64_t N, int64_t K, int64_t group_size, int dtype, void* stream) {
  B2_CHECK_ARG(weight && scales && out, B2_ERR_INVALID, "int4_dequant: null pointer");
  B2_CHECK_ARG(N > 0 && K > 0 && K % 8 == 0 && group_size > 0 && K % group_size == 0, B2_ERR_INVALID,
               "int4_dequant: bad shape N=%lld K=%lld G=%lld", (long long)N, (long long)K, (long long)group_size);
  B2_CHECK_ARG(dtype == B2_F16 || dtype == B2_BF16, B2_ERR_DTYPE, "int4_dequant: dtype %d unsupported", dtype);
  B2_CHECK_ARG(K * N < (1ll << 31), B2_ERR_UNSUPPORTED, "int4_dequant: too large");
  const int blocks = (int)((K * N + 255) / 256);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == B2_F16)
    w4_dequant_kernel<B2_F16><<<blocks, 256, 0, st>>>((const uint32_t*)weight, (const uint16_t*)scales,
                                                      (const uint16_t*)zeros, out, N, K, group_size);
  else
    w4_dequant_kernel<B2_BF16><<<blocks, 256, 0, st>>>((const uint32_t*)weight, (const uint16_t*)scales,
                                                       (const uint16_t*)zeros, out, N, K, group_size);
  return launch_status("w4_dequant");
}

extern "C" int b2_int4_repack_ref_to_gptq(const void* ref_weight, void* gptq_weight, int64_t N, int64_t K,
                                          void* stream) {
  B2_CHECK_ARG(ref_weight && gptq_weight, B2_ERR_INVALID, "int4_repack: null pointer");
  B2_CHECK_ARG(N > 0 && K > 0 && K % 8 == 0, B2_ERR_INVALID, "int4_repack: K=%lld must be a multiple of 8",
               (long long)K);
  B2_CHECK_ARG(aligned(ref_weight, 4) && aligned(gptq_weight, 4), B2_ERR_ALIGN, "int4_repack: unaligned");
  const long total = (K / 8) * N;
  w4_repack_kernel<<<(int)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint8_t*)ref_weight, (uint32_t*)gptq_weight, N, K);
  return launch_status("w4_repack");
}

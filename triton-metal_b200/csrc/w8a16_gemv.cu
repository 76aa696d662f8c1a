// W8A16 per-channel weight-only matmul: decode GEMV (M <= 16) and a generic
// per-output kernel for other shapes until the tcgen05 GEMM covers them.
//
// Math (reference int8_matmul, triton_metal/codegen/_msl_templates.py:2663-2677):
//   out[m,n] = sum_k x[m,k] * (w8[n,k] - z[n]) * s[n]
//            = s[n] * (sum_k x[m,k] w8[n,k] - z[n] * sum_k x[m,k])
//
// GEMV design: the weight [N, K] is K-major, the natural A operand of
// mma.sync m16n8k16 (rows = 16 output columns, cols = 16 k).  Lane
// (g = lane/4, t = lane%4) loads 16 k of rows g and g+8 with two 128-bit
// loads (a warp step = 16 rows x 64 k, 64 contiguous bytes per row).  Within
// each MMA, lane t's k slots are 4 consecutive bytes of its word, so x is
// consumed as plain 32-bit pairs with no permutation.  int8 -> fp16 uses the
// magic-exponent trick on (b ^ 0x80); int8 -> bf16 goes through fp32 (the
// bf16 mantissa cannot hold 128 + 255 exactly).  All K accumulates in fp32
// and the per-channel scale/zero is applied once at the end.
#include "b2_common.cuh"

namespace b2 {

constexpr int kW8Warps = 8;
constexpr int kW8Rows = 16;  // output columns per CTA
constexpr int kW8Unroll = 4;

template <int DT>
__device__ __forceinline__ void int8x4_to_pairs(uint32_t w, uint32_t& lo, uint32_t& hi) {
  if constexpr (DT == B2_F16) {
    const uint32_t u = w ^ 0x80808080u;
    lo = sub2<DT>(prmt(u, 0x64646464u, 0x4140), 0x64806480u);  // 1024 + u - 1152
    hi = sub2<DT>(prmt(u, 0x64646464u, 0x4342), 0x64806480u);
  } else {
    const uint32_t u = w ^ 0x80808080u;
    // 2^23 + u as fp32, minus 2^23 + 128 -> exact signed value
    float f0 = __uint_as_float(prmt(u, 0x4B000000u, 0x7650)) - 8388736.f;
    float f1 = __uint_as_float(prmt(u, 0x4B000000u, 0x7651)) - 8388736.f;
    float f2 = __uint_as_float(prmt(u, 0x4B000000u, 0x7652)) - 8388736.f;
    float f3 = __uint_as_float(prmt(u, 0x4B000000u, 0x7653)) - 8388736.f;
    __nv_bfloat162 a = __floats2bfloat162_rn(f0, f1), b = __floats2bfloat162_rn(f2, f3);
    lo = *reinterpret_cast<uint32_t*>(&a);
    hi = *reinterpret_cast<uint32_t*>(&b);
  }
}

template <int DT>
__device__ __forceinline__ float sum8(const uint4& v) {
  using T2 = typename dtype_of<DT>::T2;
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    T2 h = *reinterpret_cast<const T2*>(&w[i]);
    float2 f;
    if constexpr (DT == B2_F16) f = __half22float2(h); else f = __bfloat1622float2(h);
    s += f.x + f.y;
  }
  return s;
}

template <int DT, int NT, bool ZEROS>
__global__ void __launch_bounds__(kW8Warps * 32)
w8_gemv_kernel(const uint16_t* __restrict__ x, const int8_t* __restrict__ w, uint16_t* __restrict__ out,
               const uint16_t* __restrict__ scales, const uint16_t* __restrict__ zeros, int M, int N, int K) {
  using T = typename dtype_of<DT>::T;
  __shared__ float red[kW8Warps][NT * 8 * kW8Rows];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int n0 = blockIdx.x * kW8Rows;
  const int nsteps = K / 64;
  const int per_warp = (nsteps + kW8Warps - 1) / kW8Warps;
  const int s_begin = warp * per_warp, s_end = min(nsteps, s_begin + per_warp);
  const bool r0ok = n0 + g < N, r1ok = n0 + g + 8 < N;
  const int8_t* w0 = w + (size_t)(n0 + g) * K + 16 * t;
  const int8_t* w1 = w + (size_t)(n0 + g + 8) * K + 16 * t;

  float acc[NT][4];
#pragma unroll
  for (int b = 0; b < NT; ++b)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[b][c] = 0.f;
  float xs[NT];
#pragma unroll
  for (int b = 0; b < NT; ++b) xs[b] = 0.f;

  for (int s0 = s_begin; s0 < s_end; s0 += kW8Unroll) {
    uint4 wa[kW8Unroll], wb[kW8Unroll];
#pragma unroll
    for (int u = 0; u < kW8Unroll; ++u) {
      const bool ok = s0 + u < s_end;
      const size_t off = (size_t)(s0 + u) * 64;
      wa[u] = (ok && r0ok) ? ld_stream_u4(w0 + off) : make_uint4(0, 0, 0, 0);
      wb[u] = (ok && r1ok) ? ld_stream_u4(w1 + off) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kW8Unroll; ++u) {
      if (s0 + u >= s_end) break;
      const int kb = (s0 + u) * 64 + 16 * t;
      uint4 xv[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int m = g + 8 * nt;
        if (m < M) {
          const uint4* xp = reinterpret_cast<const uint4*>(x + (size_t)m * K + kb);
          xv[nt][0] = __ldg(xp);
          xv[nt][1] = __ldg(xp + 1);
        } else {
          xv[nt][0] = xv[nt][1] = make_uint4(0, 0, 0, 0);
        }
        if constexpr (ZEROS) xs[nt] += sum8<DT>(xv[nt][0]) + sum8<DT>(xv[nt][1]);
      }
      const uint32_t ra[4] = {wa[u].x, wa[u].y, wa[u].z, wa[u].w};
      const uint32_t rb[4] = {wb[u].x, wb[u].y, wb[u].z, wb[u].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t a[4];
        int8x4_to_pairs<DT>(ra[i], a[0], a[2]);
        int8x4_to_pairs<DT>(rb[i], a[1], a[3]);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint4& xq = xv[nt][i >> 1];
          const uint32_t b[2] = {(i & 1) ? xq.z : xq.x, (i & 1) ? xq.w : xq.y};
          mma_16816<DT>(acc[nt], a, b);
        }
      }
    }
  }
  // acc[nt]: c0,c1 = (n = g, m = 8nt+2t, +1); c2,c3 = (n = g+8, same m)
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int m = nt * 8 + 2 * t;
    red[warp][m * kW8Rows + g] = acc[nt][0];
    red[warp][(m + 1) * kW8Rows + g] = acc[nt][1];
    red[warp][m * kW8Rows + g + 8] = acc[nt][2];
    red[warp][(m + 1) * kW8Rows + g + 8] = acc[nt][3];
  }
  __shared__ float xsum_s[kW8Warps][16];
  if constexpr (ZEROS) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float tot = xs[nt];
      tot += __shfl_xor_sync(0xffffffffu, tot, 1);
      tot += __shfl_xor_sync(0xffffffffu, tot, 2);
      if (t == 0) xsum_s[warp][g + 8 * nt] = tot;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < NT * 8 * kW8Rows; i += blockDim.x) {
    const int m = i / kW8Rows, r = i % kW8Rows, n = n0 + r;
    if (m >= M || n >= N) continue;
    float sum = 0.f, xsum = 0.f;
#pragma unroll
    for (int ww = 0; ww < kW8Warps; ++ww) {
      sum += red[ww][i];
      if constexpr (ZEROS) xsum += xsum_s[ww][m];
    }
    const float s = to_f32<T>(*reinterpret_cast<const T*>(scales + n));
    float v;
    if constexpr (ZEROS) v = s * (sum - to_f32<T>(*reinterpret_cast<const T*>(zeros + n)) * xsum);
    else v = s * sum;
    T r16 = from_f32<T>(v);
    out[(size_t)m * N + n] = *reinterpret_cast<uint16_t*>(&r16);
  }
}

template <int DT>
__global__ void w8_generic_kernel(const uint16_t* __restrict__ x, const int8_t* __restrict__ w,
                                  uint16_t* __restrict__ out, const uint16_t* __restrict__ scales,
                                  const uint16_t* __restrict__ zeros, int M, int N, int K) {
  using T = typename dtype_of<DT>::T;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)M * N) return;
  const int m = idx / N, n = idx % N;
  float acc = 0.f, xs = 0.f;
  for (int k = 0; k < K; ++k) {
    const float xv = to_f32<T>(*reinterpret_cast<const T*>(x + (size_t)m * K + k));
    acc += xv * (float)w[(size_t)n * K + k];
    xs += xv;
  }
  const float s = to_f32<T>(*reinterpret_cast<const T*>(scales + n));
  const float z = zeros ? to_f32<T>(*reinterpret_cast<const T*>(zeros + n)) : 0.f;
  T r = from_f32<T>(s * (acc - z * xs));
  out[idx] = *reinterpret_cast<uint16_t*>(&r);
}

template <int DT>
static int w8_dispatch(const void* x, const void* w, void* out, const void* s, const void* z,
                       int M, int N, int K, cudaStream_t st) {
  dim3 grid((N + kW8Rows - 1) / kW8Rows);
  auto X = (const uint16_t*)x;
  auto W = (const int8_t*)w;
  auto O = (uint16_t*)out;
  auto S = (const uint16_t*)s;
  auto Z = (const uint16_t*)z;
  if (M <= 8) {
    if (z) w8_gemv_kernel<DT, 1, true><<<grid, kW8Warps * 32, 0, st>>>(X, W, O, S, Z, M, N, K);
    else w8_gemv_kernel<DT, 1, false><<<grid, kW8Warps * 32, 0, st>>>(X, W, O, S, Z, M, N, K);
  } else {
    if (z) w8_gemv_kernel<DT, 2, true><<<grid, kW8Warps * 32, 0, st>>>(X, W, O, S, Z, M, N, K);
    else w8_gemv_kernel<DT, 2, false><<<grid, kW8Warps * 32, 0, st>>>(X, W, O, S, Z, M, N, K);
  }
  return launch_status("w8_gemv");
}

}  // namespace b2

using namespace b2;

// Implemented in wxa16_gemm_sm100.cu: tcgen05 prefill GEMM for M > 16.
int b2_detail_w8_gemm(const void* x, const void* w, void* out, const void* s, const void* z,
                      int64_t M, int64_t N, int64_t K, int dtype, cudaStream_t st);

namespace b2 {
// quant_f32.cu: fp32 activations / scales / zeros / output on CUDA cores
int b2_detail_quant_f32(int layout, const void* x, const void* w, void* out, const void* s, const void* z,
                        int64_t M, int64_t N, int64_t K, int64_t G, cudaStream_t st);
}  // namespace b2

extern "C" int b2_int8_matmul(const void* input, const void* weight, void* output,
                              const void* scales, const void* zeros,
                              int64_t M, int64_t N, int64_t K, int dtype, void* stream) {
  B2_CHECK_ARG(input && weight && output && scales, B2_ERR_INVALID, "int8_matmul: null pointer");
  B2_CHECK_ARG(M >= 0 && N > 0 && K > 0, B2_ERR_INVALID, "int8_matmul: bad shape M=%lld N=%lld K=%lld",
               (long long)M, (long long)N, (long long)K);
  B2_CHECK_ARG(dtype == B2_F16 || dtype == B2_BF16 || dtype == B2_F32, B2_ERR_DTYPE,
               "int8_matmul: dtype %d unsupported", dtype);
  B2_CHECK_ARG(M * N < (1ll << 31) && N * K < (1ll << 40), B2_ERR_UNSUPPORTED, "int8_matmul: too large");
  if (M == 0) return B2_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == B2_F32) return b2_detail_quant_f32(2, input, weight, output, scales, zeros, M, N, K, 0, st);
  const bool fast = M <= 16 && K % 64 == 0 && aligned(input, 16) && aligned(weight, 16);
  if (fast)
    return dtype == B2_F16 ? w8_dispatch<B2_F16>(input, weight, output, scales, zeros, M, N, K, st)
                           : w8_dispatch<B2_BF16>(input, weight, output, scales, zeros, M, N, K, st);
  if (M > 16) {
    int r = b2_detail_w8_gemm(input, weight, output, scales, zeros, M, N, K, dtype, st);
    if (r != B2_ERR_UNSUPPORTED) return r;
  }
  const int blocks = (int)((M * N + 255) / 256);
  if (dtype == B2_F16)
    w8_generic_kernel<B2_F16><<<blocks, 256, 0, st>>>((const uint16_t*)input, (const int8_t*)weight,
                                                      (uint16_t*)output, (const uint16_t*)scales,
                                                      (const uint16_t*)zeros, M, N, K);
  else
    w8_generic_kernel<B2_BF16><<<blocks, 256, 0, st>>>((const uint16_t*)input, (const int8_t*)weight,
                                                       (uint16_t*)output, (const uint16_t*)scales,
                                                       (const uint16_t*)zeros, M, N, K);
  return launch_status("w8_generic");
}

// W4A16 in the reference's own weight layout, natively (no repack):
//   weight uint8 [N, K/2], byte j of row n = k 2j (low nibble), 2j+1 (high)
//   scales, zeros [N, K/G] (activation dtype)
// (reference int4_matmul, triton_metal/codegen/_msl_templates.py:2682-2745;
// nibble order :2725-2732, buffers :2705-2712).
//
// b2_int4_matmul_ref: M <= 16 -> the decode GEMV below; M > 16 -> the
// tcgen05 prefill GEMM (wxa16_gemm_sm100.cu, MODE 3); other shapes -> a
// generic per-output kernel.
//
// GEMV design: the weight is K-major, the natural A operand of mma.sync
// m16n8k16 (rows = 16 output columns).  One CTA owns 16 rows; its 8 warps
// split K in steps of 128 k.  Lane (g = lane/4, t = lane%4) loads 16
// contiguous bytes (32 k) of rows g and g+8 per step; each 32-bit word is 8
// consecutive k = 4 bytes = 4 k-ordered pairs, so a word feeds two MMAs
// (pairs 0,1 then 2,3) with x read in its natural order (8 halves per word).
// The group scale (and zero) is folded into the 16-bit operand:
// (q - 8) s, or (q - zi) s - zf s with zi = rint(z), one rounding per value,
// so MMAs accumulate across groups with no per-group combine.
#include "b2_common.cuh"

namespace b2 {
namespace w4ref {

constexpr int kWarps = 8;
constexpr int kRows = 16;    // output columns per CTA
constexpr int kUnroll = 2;   // 128-k steps in flight per warp

template <int DT>
__device__ __forceinline__ uint32_t splat2(float v) {
  if constexpr (DT == B2_BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v, v);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(v, v);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// group constants of one row: scale pair, exact bias pair (bias + zi) and
// the residual pair -zf * s (zero when symmetric: zi = 8)
template <int DT, bool ZP>
__device__ __forceinline__ void group_consts(const uint16_t* scales, const uint16_t* zeros, size_t gi, bool ok,
                                             uint32_t& s2, uint32_t& bz2, uint32_t& zr2) {
  using T = typename dtype_of<DT>::T;
  const float bias = DT == B2_BF16 ? 128.f : 1024.f;
  const float sc = ok ? to_f32<T>(*reinterpret_cast<const T*>(scales + gi)) : 0.f;
  s2 = splat2<DT>(sc);
  if constexpr (ZP) {
    const float z = ok ? to_f32<T>(*reinterpret_cast<const T*>(zeros + gi)) : 0.f;
    const float zi = fminf(fmaxf(rintf(z), -64.f), 64.f);
    bz2 = splat2<DT>(bias + zi);
    zr2 = splat2<DT>(-(z - zi) * sc);
  } else {
    bz2 = splat2<DT>(bias + 8.f);
    zr2 = 0u;
  }
}

// pair j (k = 2j, 2j+1 of the word) -> (q - zi) s + zr, 16-bit pair
template <int DT>
__device__ __forceinline__ uint32_t dq_pair(uint32_t w, uint32_t w4, int j, uint32_t s2, uint32_t bz2,
                                            uint32_t zr2) {
  constexpr uint32_t kBias = DT == B2_BF16 ? 0x43004300u : 0x64006400u;
  const uint32_t biased = and_or(prmt(w, w4, (uint32_t)(j | ((4 + j) << 8))), 0x000F000Fu, kBias);
  const uint32_t v = sub2<DT>(biased, bz2);  // q - zi, exact
  uint32_t r;
  if constexpr (DT == B2_BF16) asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(v), "r"(s2), "r"(zr2));
  else asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(v), "r"(s2), "r"(zr2));
  return r;
}

template <int DT, int NT, bool ZP>
__global__ void __launch_bounds__(kWarps * 32)
w4ref_gemv_kernel(const uint16_t* __restrict__ x, const uint8_t* __restrict__ w, uint16_t* __restrict__ out,
                  const uint16_t* __restrict__ scales, const uint16_t* __restrict__ zeros, int M, int N, int K,
                  int G) {
  using T = typename dtype_of<DT>::T;
  __shared__ float red[kWarps][NT * 8 * kRows];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int n0 = blockIdx.x * kRows;
  const int nsteps = K / 128;
  const int per_warp = (nsteps + kWarps - 1) / kWarps;
  const int s_begin = warp * per_warp, s_end = min(nsteps, s_begin + per_warp);
  const bool r0ok = n0 + g < N, r1ok = n0 + g + 8 < N;
  const size_t rb = (size_t)K / 2;  // bytes per weight row
  const uint8_t* w0 = w + (size_t)(n0 + g) * rb + 16 * t;
  const uint8_t* w1 = w + (size_t)(n0 + g + 8) * rb + 16 * t;
  const int ng = K / G;

  float acc[2][NT][4];
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int b = 0; b < NT; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;

  for (int s0 = s_begin; s0 < s_end; s0 += kUnroll) {
    uint4 wa[kUnroll], wb[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const bool ok = s0 + u < s_end;
      const size_t off = (size_t)(s0 + u) * 64;
      wa[u] = (ok && r0ok) ? ld_stream_u4(w0 + off) : make_uint4(0, 0, 0, 0);
      wb[u] = (ok && r1ok) ? ld_stream_u4(w1 + off) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (s0 + u >= s_end) break;
      const int kb = (s0 + u) * 128 + 32 * t;  // this lane's 32 k (one group: G % 32 == 0)
      const int grp = kb / G;
      uint32_t sa, ba, za, sb, bb, zb;
      group_consts<DT, ZP>(scales, zeros, (size_t)(n0 + g) * ng + grp, r0ok, sa, ba, za);
      group_consts<DT, ZP>(scales, zeros, (size_t)(n0 + g + 8) * ng + grp, r1ok, sb, bb, zb);
      const uint32_t ra[4] = {wa[u].x, wa[u].y, wa[u].z, wa[u].w};
      const uint32_t rbw[4] = {wb[u].x, wb[u].y, wb[u].z, wb[u].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 xv[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int m = g + 8 * nt;
          xv[nt] = m < M ? __ldg(reinterpret_cast<const uint4*>(x + (size_t)m * K + kb + 8 * i))
                         : make_uint4(0, 0, 0, 0);
        }
        const uint32_t a4 = ra[i] >> 4, b4 = rbw[i] >> 4;
        // MMA 1: pairs 0 (slots 2t, 2t+1) and 1 (slots 2t+8, 2t+9); MMA 2: pairs 2, 3
        const uint32_t A1[4] = {dq_pair<DT>(ra[i], a4, 0, sa, ba, za), dq_pair<DT>(rbw[i], b4, 0, sb, bb, zb),
                                dq_pair<DT>(ra[i], a4, 1, sa, ba, za), dq_pair<DT>(rbw[i], b4, 1, sb, bb, zb)};
        const uint32_t A2[4] = {dq_pair<DT>(ra[i], a4, 2, sa, ba, za), dq_pair<DT>(rbw[i], b4, 2, sb, bb, zb),
                                dq_pair<DT>(ra[i], a4, 3, sa, ba, za), dq_pair<DT>(rbw[i], b4, 3, sb, bb, zb)};
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint32_t b1[2] = {xv[nt].x, xv[nt].y};  // k + 0..3
          const uint32_t b2[2] = {xv[nt].z, xv[nt].w};  // k + 4..7
          mma_16816<DT>(acc[i & 1][nt], A1, b1);
          mma_16816<DT>(acc[i & 1][nt], A2, b2);
        }
      }
    }
  }
  // acc[.][nt]: c0,c1 = (n = g, m = 8nt+2t, +1); c2,c3 = (n = g+8, same m)
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int m = nt * 8 + 2 * t;
    red[warp][m * kRows + g] = acc[0][nt][0] + acc[1][nt][0];
    red[warp][(m + 1) * kRows + g] = acc[0][nt][1] + acc[1][nt][1];
    red[warp][m * kRows + g + 8] = acc[0][nt][2] + acc[1][nt][2];
    red[warp][(m + 1) * kRows + g + 8] = acc[0][nt][3] + acc[1][nt][3];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < NT * 8 * kRows; i += blockDim.x) {
    const int m = i / kRows, r = i % kRows, n = n0 + r;
    if (m >= M || n >= N) continue;
    float sum = 0.f;
#pragma unroll
    for (int ww = 0; ww < kWarps; ++ww) sum += red[ww][i];
    T r16 = from_f32<T>(sum);
    out[(size_t)m * N + n] = *reinterpret_cast<uint16_t*>(&r16);
  }
}

// One thread per output, any shape: out[m, n] = sum_k x (q - z) s in fp32.
template <int DT>
__global__ void w4ref_generic_kernel(const uint16_t* __restrict__ x, const uint8_t* __restrict__ w,
                                     uint16_t* __restrict__ out, const uint16_t* __restrict__ scales,
                                     const uint16_t* __restrict__ zeros, int M, int N, int K, int G) {
  using T = typename dtype_of<DT>::T;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)M * N) return;
  const int m = idx / N, n = idx % N, ng = (K + G - 1) / G;
  float acc = 0.f;
  for (int k = 0; k < K; ++k) {
    const uint8_t byte = w[(size_t)n * ((K + 1) / 2) + k / 2];
    const int q = (k & 1) ? (byte >> 4) & 0xF : byte & 0xF;
    const size_t gi = (size_t)n * ng + k / G;
    const float s = to_f32<T>(*reinterpret_cast<const T*>(scales + gi));
    const float z = zeros ? to_f32<T>(*reinterpret_cast<const T*>(zeros + gi)) : 8.f;
    acc += to_f32<T>(*reinterpret_cast<const T*>(x + (size_t)m * K + k)) * ((float)q - z) * s;
  }
  T r = from_f32<T>(acc);
  out[idx] = *reinterpret_cast<uint16_t*>(&r);
}

}  // namespace w4ref
}  // namespace b2

using namespace b2;

// Implemented in wxa16_gemm_sm100.cu: tcgen05 prefill GEMM, reference layout.
int b2_detail_w4_gemm_ref(const void* x, const void* w, void* out, const void* s, const void* z, int64_t M,
                          int64_t N, int64_t K, int64_t G, int dtype, cudaStream_t st);

namespace b2 {
// quant_f32.cu: fp32 activations / scales / zeros / output on CUDA cores
int b2_detail_quant_f32(int layout, const void* x, const void* w, void* out, const void* s, const void* z,
                        int64_t M, int64_t N, int64_t K, int64_t G, cudaStream_t st);
}  // namespace b2

extern "C" int b2_int4_matmul_ref(const void* input, const void* weight, void* output, const void* scales,
                                  const void* zeros, int64_t M, int64_t N, int64_t K, int64_t group_size, int dtype,
                                  void* stream) {
  B2_CHECK_ARG(input && weight && output && scales, B2_ERR_INVALID, "int4_matmul_ref: null pointer");
  B2_CHECK_ARG(M >= 0 && N > 0 && K > 0 && group_size > 0, B2_ERR_INVALID, "int4_matmul_ref: bad shape");
  B2_CHECK_ARG(dtype == B2_F16 || dtype == B2_BF16 || dtype == B2_F32, B2_ERR_DTYPE,
               "int4_matmul_ref: dtype %d unsupported", dtype);
  B2_CHECK_ARG(M * N < (1ll << 31) && N * K / 2 < (1ll << 31), B2_ERR_UNSUPPORTED, "int4_matmul_ref: too large");
  if (M == 0) return B2_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == B2_F32) return b2_detail_quant_f32(1, input, weight, output, scales, zeros, M, N, K, group_size, st);
  const auto X = (const uint16_t*)input;
  const auto W = (const uint8_t*)weight;
  const auto O = (uint16_t*)output;
  const auto S = (const uint16_t*)scales;
  const auto Z = (const uint16_t*)zeros;
  const bool fast = K % 128 == 0 && group_size % 32 == 0 && K % group_size == 0 && aligned(input, 16) &&
                    aligned(weight, 16);
  if (M <= 16 && fast) {
    const dim3 grid((unsigned)((N + w4ref::kRows - 1) / w4ref::kRows));
    const int t = w4ref::kWarps * 32;
#define B2_W4R(DT, NT)                                                                                         \
  do {                                                                                                         \
    if (Z) w4ref::w4ref_gemv_kernel<DT, NT, true><<<grid, t, 0, st>>>(X, W, O, S, Z, (int)M, (int)N, (int)K,   \
                                                                         (int)group_size);                     \
    else w4ref::w4ref_gemv_kernel<DT, NT, false><<<grid, t, 0, st>>>(X, W, O, S, Z, (int)M, (int)N, (int)K,    \
                                                                        (int)group_size);                      \
  } while (0)
    if (dtype == B2_F16) {
      if (M <= 8) B2_W4R(B2_F16, 1); else B2_W4R(B2_F16, 2);
    } else {
      if (M <= 8) B2_W4R(B2_BF16, 1); else B2_W4R(B2_BF16, 2);
    }
#undef B2_W4R
    return launch_status("w4ref_gemv");
  }
  if (M > 16) {
    const int r = b2_detail_w4_gemm_ref(input, weight, output, scales, zeros, M, N, K, group_size, dtype, st);
    if (r != B2_ERR_UNSUPPORTED) return r;
  }
  const long total = M * N;
  const int blocks = (int)((total + 255) / 256);
  if (dtype == B2_F16)
    w4ref::w4ref_generic_kernel<B2_F16><<<blocks, 256, 0, st>>>(X, W, O, S, Z, (int)M, (int)N, (int)K,
                                                                (int)group_size);
  else
    w4ref::w4ref_generic_kernel<B2_BF16><<<blocks, 256, 0, st>>>(X, W, O, S, Z, (int)M, (int)N, (int)K,
                                                                 (int)group_size);
  return launch_status("w4ref_generic");
}

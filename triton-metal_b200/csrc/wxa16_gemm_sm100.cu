// Prefill GEMM on the 5th-generation tensor cores (tcgen05, sm_100a):
//   out[M, N] (bf16) = x[M, K] (bf16) @ W[K, N]
// with W given as
//   MODE 0: bf16 [N, K] (K-major, nn.Linear layout)       -> b2_gemm_bf16
//   MODE 1: int8 [N, K] + per-channel scale [N]            -> b2_int8_matmul
//           (reference int8_matmul, _msl_templates.py:2663-2677)
//   MODE 2: int4 GPTQ int32 [K/8, N] + group scales [K/G, N] (zero point 8)
//                                                          -> b2_int4_matmul
//           (reference int4_matmul, _msl_templates.py:2716-2743)
//
// Persistent, warp-specialised CTA (one per SM), tile 128 x 256 x 64:
//   warp 0      TMA producer: x tile (and W tile / packed W tile) per k-block
//               into a ring of shared-memory stages (128B-swizzled, no
//               multicast);
//   warp 1      TMEM owner + MMA issuer: one thread issues 4 x
//               tcgen05.mma (M=128, N=256, K=16) per k-block into a TMEM
//               accumulator (2 x 256 columns, double-buffered across tiles)
//               and commits the stage back to the producer;
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns, (per-channel
//               scale), bf16 convert, global store; frees the accumulator;
//   warps 6-21  (MODE 1/2) dequantisers: packed tile -> exact integers ->
//               scaled bf16 written straight into the 128B-swizzled K-major
//               B layout the MMA reads, then fence.proxy.async + arrive.
// All waits are bounded (error word + early exit).
#include "tc_common.cuh"
#include <string.h>

namespace b2 {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int kABytes = BM * BK * 2;   // 16 KB
constexpr int kBBytes = BN * BK * 2;   // 32 KB
constexpr int kAccCols = BN;           // fp32 accumulator columns per buffer
constexpr int kTmemCols = 2 * kAccCols;
constexpr int kDequantWarps = 16;

template <int MODE>
struct Cfg {
  static constexpr int kPackedBytes = MODE == 0 ? 0 : (MODE == 1 ? BN * BK : (BK / 8) * BN * 4);
  static constexpr int kStageBytes = kABytes + kBBytes + kPackedBytes;
  static constexpr int kStages = (220 * 1024) / kStageBytes;
  static constexpr int kWarps = MODE == 0 ? 6 : 6 + kDequantWarps;
  static constexpr int kThreads = kWarps * 32;
  static constexpr size_t kSmem = (size_t)kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

struct Params {
  int M, N, K, G;
  const __nv_bfloat16* scales;  // MODE 1: [N]; MODE 2: [K/G, N]
  __nv_bfloat16* out;
  int tiles_m, tiles_n;
  unsigned* err;
};

// Bounded wait that also gives up when another role already aborted.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, const Params& p, unsigned code,
                                              volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitNs) break;
    }
  }
  atomicCAS(p.err, 0u, code);
  *abort_flag = 1;
  return false;
}

// int4 word (k = 8r..8r+7 in nibbles 0..7) -> nibble order 0,2,4,6,1,3,5,7 so
// that (w >> 4j) & 0x000F000F holds the adjacent pair (k = 2j, 2j+1).
__device__ __forceinline__ uint32_t unzip_nibbles(uint32_t w) {
  uint32_t t = ((w >> 4) ^ w) & 0x00F000F0u;  // swap nibbles 1<->2 in each half
  w ^= t ^ (t << 4);
  return prmt(w, w, 0x3120);                 // bytes (q0q2)(q1q3)(q4q6)(q5q7) -> (q0q2)(q4q6)(q1q3)(q5q7)
}

// 8 k-values of one column -> 4 packed bf16 pairs of (q - 8) * s.
__device__ __forceinline__ uint4 dequant8_int4(uint32_t w, uint32_t s2) {
  const uint32_t u = unzip_nibbles(w);
  uint32_t r[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t v = sub2<B2_BF16>(and_or(u >> (4 * j), 0x000F000Fu, 0x43004300u), 0x43084308u);  // q - 8, exact
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r[j]) : "r"(v), "r"(s2));
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

// 4 int8 -> 2 packed bf16 pairs (exact).
__device__ __forceinline__ void int8x4_to_bf16(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  const float f0 = __uint_as_float(prmt(u, 0x4B000000u, 0x7650)) - 8388736.f;
  const float f1 = __uint_as_float(prmt(u, 0x4B000000u, 0x7651)) - 8388736.f;
  const float f2 = __uint_as_float(prmt(u, 0x4B000000u, 0x7652)) - 8388736.f;
  const float f3 = __uint_as_float(prmt(u, 0x4B000000u, 0x7653)) - 8388736.f;
  __nv_bfloat162 a = __floats2bfloat162_rn(f0, f1), b = __floats2bfloat162_rn(f2, f3);
  lo = *reinterpret_cast<uint32_t*>(&a);
  hi = *reinterpret_cast<uint32_t*>(&b);
}

template <int MODE>
__global__ void __launch_bounds__(Cfg<MODE>::kThreads, 1)
wxa16_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const Params p) {
  using C = Cfg<MODE>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sA = smem;
  uint8_t* sB = sA + C::kStages * kABytes;
  uint8_t* sP = sB + C::kStages * kBBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sP + C::kStages * C::kPackedBytes);
  uint64_t* bready = full + C::kStages;
  uint64_t* empty = bready + C::kStages;
  uint64_t* tfull = empty + C::kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kblocks = p.K / BK;
  const int ntiles = p.tiles_m * p.tiles_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&bready[s], kDequantWarps);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_holder, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int m0 = (tile % p.tiles_m) * BM, n0 = (tile / p.tiles_m) * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_or_abort(&empty[stage], phase ^ 1, p, 0xB2100001u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t bytes = kABytes + (MODE == 0 ? kBBytes : C::kPackedBytes);
          mbar_arrive_expect_tx(&full[stage], bytes);
          tma_load_2d(sA + stage * kABytes, &tmA, kb * BK, m0, &full[stage]);
          if constexpr (MODE == 0) tma_load_2d(sB + stage * kBBytes, &tmB, kb * BK, n0, &full[stage]);
          if constexpr (MODE == 1) tma_load_2d(sP + stage * C::kPackedBytes, &tmB, kb * BK, n0, &full[stage]);
          if constexpr (MODE == 2) tma_load_2d(sP + stage * C::kPackedBytes, &tmB, n0, kb * (BK / 8), &full[stage]);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_f16(BM, BN, true);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!wait_or_abort(&tempty[acc], acc_phase ^ 1, p, 0xB2100002u, abort_flag)) break;
        tc::fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * kAccCols;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_or_abort(&full[stage], phase, p, 0xB2100003u, abort_flag) ||
              (MODE != 0 && !wait_or_abort(&bready[stage], phase, p, 0xB2100004u, abort_flag))) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint64_t da = tc::desc_kmajor_sw128(sA + stage * kABytes);
          const uint64_t db = tc::desc_kmajor_sw128(sB + stage * kBBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // +32 bytes of K per step inside the 128-byte swizzled row
            tc::mma_f16_ss(d_tmem, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, (kb | k) != 0);
          }
          tc::commit(&empty[stage]);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) tc::commit(&tfull[acc]);
      }
      if (!ok) {
        // aborted: let every MMA already issued finish before TMEM is freed
        tc::commit(drain);
        mbar_wait(drain, 0, p.err, 0xB2100007u);
      }
    }
  } else if (warp < 6) {
    // ------------------------------ epilogue ----------------------------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int it = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
      const int m0 = (tile % p.tiles_m) * BM, n0 = (tile / p.tiles_m) * BN;
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!wait_or_abort(&tfull[acc], acc_phase, p, 0xB2100005u, abort_flag)) break;
      tc::fence_after_sync();
      const int row = m0 + q * 32 + lane;
      __nv_bfloat16* orow = p.out + (size_t)row * p.N + n0;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tc::tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + acc * kAccCols + c * 32, r);
        tc::tmem_ld_wait();
        uint32_t packed[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float v0 = __uint_as_float(r[2 * j]), v1 = __uint_as_float(r[2 * j + 1]);
          if constexpr (MODE == 1) {
            const int n = n0 + c * 32 + 2 * j;
            v0 *= __bfloat162float(p.scales[n]);
            v1 *= __bfloat162float(p.scales[n + 1]);
          }
          __nv_bfloat162 h = __floats2bfloat162_rn(v0, v1);
          packed[j] = *reinterpret_cast<uint32_t*>(&h);
        }
        uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          dst[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  } else if constexpr (MODE != 0) {
    // ------------------------------ dequantisers ------------------------------
    const int d = (warp - 6) * 32 + lane;
    const int n = d & (BN - 1);  // B row (output column) this thread fills
    const int h = d / BN;        // which half of the row's 64 k
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
      const int n0 = (tile / p.tiles_m) * BN;
      uint32_t s2 = 0;
      int cur_group = -1;
      for (int kb = 0; kb < kblocks; ++kb) {
        if (MODE == 2) {
          const int grp = kb * BK / p.G;
          if (grp != cur_group) {
            const __nv_bfloat16 s = p.scales[(size_t)grp * p.N + n0 + n];
            __nv_bfloat162 ss = __halves2bfloat162(s, s);
            s2 = *reinterpret_cast<uint32_t*>(&ss);
            cur_group = grp;
          }
        }
        if (!wait_or_abort(&full[stage], phase, p, 0xB2100006u, abort_flag)) {
          ok = false;
          break;
        }
        uint8_t* brow = sB + stage * kBBytes + n * 128;
        const int sw = n & 7;
        if constexpr (MODE == 2) {
          const uint32_t* pk = reinterpret_cast<const uint32_t*>(sP + stage * C::kPackedBytes);
#pragma unroll
          for (int rr = 0; rr < BK / 16; ++rr) {
            const int r = h * (BK / 16) + rr;
            const uint4 v = dequant8_int4(pk[r * BN + n], s2);
            *reinterpret_cast<uint4*>(brow + ((r ^ sw) << 4)) = v;
          }
        } else {
          const uint4* pk = reinterpret_cast<const uint4*>(sP + stage * C::kPackedBytes + n * BK);
#pragma unroll
          for (int jj = 0; jj < BK / 32; ++jj) {
            const int j = h * (BK / 32) + jj;
            const uint4 v = pk[j];
            uint32_t o[8];
            int8x4_to_bf16(v.x, o[0], o[1]);
            int8x4_to_bf16(v.y, o[2], o[3]);
            int8x4_to_bf16(v.z, o[4], o[5]);
            int8x4_to_bf16(v.w, o[6], o[7]);
            *reinterpret_cast<uint4*>(brow + (((2 * j) ^ sw) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<uint4*>(brow + (((2 * j + 1) ^ sw) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
          }
        }
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bready[stage]);
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  }

  // teardown: every role is done (or aborted); free TMEM from the owner warp
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace gemm

template <int MODE>
static int launch_gemm(const void* x, const void* w, const void* scales, void* out, int64_t M, int64_t N,
                       int64_t K, int64_t G, cudaStream_t st) {
  using namespace gemm;
  using C = Cfg<MODE>;
  if (M % BM || N % BN || K % BK || (MODE == 2 && (G % BK || K % G))) return B2_ERR_UNSUPPORTED;
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(out, 16)) return B2_ERR_UNSUPPORTED;
  unsigned* err = device_error_word();
  if (!err) {
    set_error("gemm: cannot resolve the device error word");
    return B2_ERR_LAUNCH;
  }
  CUtensorMap ta, tb;
  if (!make_tmap_2d(&ta, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, K, M, K * 2, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B))
    return B2_ERR_INVALID;
  bool okb;
  if (MODE == 0)
    okb = make_tmap_2d(&tb, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, K, N, K * 2, BK, BN, CU_TENSOR_MAP_SWIZZLE_128B);
  else if (MODE == 1)
    okb = make_tmap_2d(&tb, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, N, K, BK, BN);
  else
    okb = make_tmap_2d(&tb, w, CU_TENSOR_MAP_DATA_TYPE_UINT32, N, K / 8, N * 4, BN, BK / 8);
  if (!okb) return B2_ERR_INVALID;
  Params p;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.G = (int)G;
  p.scales = (const __nv_bfloat16*)scales;
  p.out = (__nv_bfloat16*)out;
  p.tiles_m = (int)(M / BM);
  p.tiles_n = (int)(N / BN);
  p.err = err;
  const int ntiles = p.tiles_m * p.tiles_n;
  int grid = num_sms();
  if (grid > ntiles) grid = ntiles;
  auto kern = wxa16_gemm_kernel<MODE>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmem);
  kern<<<grid, C::kThreads, C::kSmem, st>>>(ta, tb, p);
  return launch_status("wxa16_gemm");
}

}  // namespace b2

using namespace b2;

// Called by b2_int4_matmul for M > 16: bf16, symmetric zero point only.
int b2_detail_w4_gemm(const void* x, const void* w, void* out, const void* s, const void* z, int64_t M, int64_t N,
                      int64_t K, int64_t G, int dtype, cudaStream_t st) {
  if (dtype != B2_BF16 || z) return B2_ERR_UNSUPPORTED;
  return launch_gemm<2>(x, w, s, out, M, N, K, G, st);
}

// Called by b2_int8_matmul for M > 16: bf16, symmetric only.
int b2_detail_w8_gemm(const void* x, const void* w, void* out, const void* s, const void* z, int64_t M, int64_t N,
                      int64_t K, int dtype, cudaStream_t st) {
  if (dtype != B2_BF16 || z) return B2_ERR_UNSUPPORTED;
  return launch_gemm<1>(x, w, s, out, M, N, K, 0, st);
}

extern "C" int b2_gemm_bf16(const void* x, const void* w, void* out, int64_t M, int64_t N, int64_t K, void* stream) {
  B2_CHECK_ARG(x && w && out, B2_ERR_INVALID, "gemm_bf16: null pointer");
  B2_CHECK_ARG(M > 0 && N > 0 && K > 0, B2_ERR_INVALID, "gemm_bf16: bad shape");
  int r = launch_gemm<0>(x, w, nullptr, out, M, N, K, 0, (cudaStream_t)stream);
  if (r == B2_ERR_UNSUPPORTED)
    set_error("gemm_bf16: needs M %% 128 == 0, N %% 256 == 0, K %% 64 == 0 and 16-byte aligned pointers");
  return r;
}

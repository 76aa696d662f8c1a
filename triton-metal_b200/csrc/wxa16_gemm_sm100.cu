// Prefill GEMM on the 5th-generation tensor cores (tcgen05, sm_100a):
//   out[M, N] = x[M, K] @ W[K, N]      (x, out: bf16 or fp16; fp32 accumulate)
// with W given as
//   MODE 0: bf16 [N, K] (K-major, nn.Linear layout)       -> b2_gemm_bf16
//   MODE 1: int8 [N, K] + per-channel scale [N] (+ zero [N]) -> b2_int8_matmul
//           (reference int8_matmul, _msl_templates.py:2663-2677)
//   MODE 2: int4 GPTQ int32 [K/8, N] + group scales [K/G, N], zero point 8 or
//           per-group zeros [K/G, N] (asymmetric)
//   MODE 3: int4 in the reference's own layout: uint8 [N, K/2], low nibble
//           = even k, scales (zeros) [N, K/G] (_msl_templates.py:2693-2695,
//           :2725-2732)                            -> b2_int4_matmul_ref
//                                                          -> b2_int4_matmul
//           (reference int4_matmul, _msl_templates.py:2716-2743)
//
// Persistent, warp-specialised CTA (one per SM), tile 128 x bn x 64 (bn <= 256
// picked per launch to fill the last round of tiles):
//   warp 0      TMA producer: x tile (and W tile / packed W tile) per k-block
//               into a ring of shared-memory stages (128B-swizzled, no
//               multicast);
//   warp 1      TMEM owner + MMA issuer: one thread issues 4 x
//               tcgen05.mma (M=128, N=256, K=16) per k-block into a TMEM
//               accumulator (2 x 256 columns, double-buffered across tiles)
//               and commits the stage back to the producer;
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns, (per-channel
//               scale), bf16 convert, 32 x 32 tile staged in shared memory
//               and written by a TMA store; frees the accumulator;
//   warps 6-21  (MODE 1/2) dequantisers: packed tile -> exact integers ->
//               scaled bf16 written straight into the 128B-swizzled K-major
//               B layout the MMA reads, then fence.proxy.async + arrive.
// M and N may be ragged (multiples of 1 and 8): the TMA boxes past the edge
// read zeros and the TMA stores clip at M / N.  All waits are bounded
// (error word + early exit).
#include "tc_common.cuh"
#include <stdlib.h>
#include <string.h>

namespace b2 {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int kBBytes = BN * BK * 2;   // 32 KB
constexpr int kAccCols = BN;           // fp32 accumulator columns per buffer
constexpr int kTmemCols = 2 * kAccCols;
constexpr int kDequantWarps = 16;
// W8 with zeros: per-tile row sums of x, [2 k-halves][256 rows] fp32
constexpr int kXsBytes = 2 * 2 * BM * 4;
// epilogue: one 32 x 32 output tile (16-bit) per epilogue warp, stored by TMA
constexpr int kEpiTile = 32 * 32 * 2;
constexpr int kEpiBytes = 4 * kEpiTile;
// W8: each epilogue warp's copy of the tile's per-channel scales and zeros
// (16-bit, [2][BN])
constexpr int kEpiSzBytes = 4 * 2 * BN * 2;

template <int MODE>
struct Cfg {
  // MODE 2 (W4): a 256-row CTA tile, two M = 128 MMAs per k-step sharing one
  // dequantised B tile (the dequant work per FLOP halves; TMEM holds the two
  // M halves instead of a double buffer): 57% -> 85% of the bf16 peak.
  // MODE 0 / 1: 128 rows, the two TMEM buffers double-buffer consecutive
  // tiles (W8 with 256 rows fits only 2 stages and measured slower).
  static constexpr bool TWO = MODE != 0;
  // W8: the dequantised B tile lives outside the stage ring, double-buffered
  // (B buffer kbi & 1 per k-block), so 3 stages of A + packed int8 fit next
  // to the 256-row A tiles (with B in the ring only 2 stages would fit)
  static constexpr bool SPLITB = MODE == 1;
  static constexpr int BMC = TWO ? 2 * BM : BM;
  static constexpr int kABytesC = BMC * BK * 2;
  static constexpr int kPackedBytes = MODE == 0 ? 0 : (MODE == 1 ? BN * BK : BN * BK / 2);
  static constexpr int kStageBytes = kABytesC + (SPLITB ? 0 : kBBytes) + kPackedBytes;
  static constexpr int kStages = SPLITB ? 3 : (220 * 1024) / kStageBytes;
  static constexpr int kBRegion = SPLITB ? 2 * kBBytes : kStages * kBBytes;
  static constexpr int kWarps = MODE == 0 ? 6 : 6 + kDequantWarps;
  static constexpr int kThreads = kWarps * 32;
  static constexpr size_t kSmem = (size_t)kStages * kStageBytes + (SPLITB ? kBRegion : 0) + 1024 /*align*/ +
                                  256 /*barriers*/ +
                                  (MODE == 1 ? kXsBytes + kEpiSzBytes : 0) + kEpiBytes;
};

static_assert(Cfg<0>::kSmem <= 227 * 1024 && Cfg<1>::kSmem <= 227 * 1024 && Cfg<2>::kSmem <= 227 * 1024 &&
                  Cfg<3>::kSmem <= 227 * 1024,
              "shared memory per CTA");

struct Params {
  int M, N, K, G;
  const uint16_t* scales;  // MODE 1: [N]; MODE 2: [K/G, N]   (activation dtype)
  const uint16_t* zeros;   // same shape as scales, or null (symmetric)
  uint16_t* out;
  int tiles_m, tiles_n;
  int bn;          // CTA tile width in columns (<= BN, multiple of 32), chosen per launch
  uint32_t idesc;  // MMA instruction descriptor for M = 128, N = bn
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

// 8 k-values of one column -> 4 packed pairs (activation dtype) of
// (q - 8) * s (symmetric) or (q - z) * s (asymmetric).  Both layouts hold the
// pair (k = 2j, 2j + 1) in byte j of a 32-bit word (low nibble, high nibble):
// a GPTQ int32 (k = 8r .. 8r + 7 in nibbles 0 .. 7) and four bytes of a
// reference [N, K/2] row.  One PRMT puts byte j of w and of w >> 4 into the
// two halves, one LOP3 keeps the nibbles and ORs in the bias (9 integer ops
// per word; a nibble unzip followed by shifts took 12 and measured 1203 TF/s
// at C2 against 1238).  q is exact: OR-ing it into the mantissa of 128.0
// (bf16, ulp 1) or 1024.0 (fp16, ulp 1) gives bias + q.  With zeros,
// z = zi + zf (zi = rint(z)): subtracting the exact pair bz2 = bias + zi
// leaves q - zi exactly, and one fma adds the small residual zr2 = -zf * s,
// so the result is rounded once (plus the rounding of the |zf| <= 1/2
// residual).
template <int DT, bool ZP>
__device__ __forceinline__ uint4 dequant8_int4(uint32_t w, uint32_t s2, uint32_t bz2, uint32_t zr2) {
  constexpr uint32_t kBias = DT == B2_BF16 ? 0x43004300u : 0x64006400u;
  constexpr uint32_t kBias8 = DT == B2_BF16 ? 0x43084308u : 0x64086408u;
  const uint32_t w4 = w >> 4;
  uint32_t r[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t biased = and_or(prmt(w, w4, (uint32_t)(j | ((4 + j) << 8))), 0x000F000Fu, kBias);
    if constexpr (!ZP) {
      const uint32_t v = sub2<DT>(biased, kBias8);
      if constexpr (DT == B2_BF16) asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r[j]) : "r"(v), "r"(s2));
      else asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r[j]) : "r"(v), "r"(s2));
    } else {
      const uint32_t v = sub2<DT>(biased, bz2);
      if constexpr (DT == B2_BF16) asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r[j]) : "r"(v), "r"(s2), "r"(zr2));
      else asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r[j]) : "r"(v), "r"(s2), "r"(zr2));
    }
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

template <int DT>
__device__ __forceinline__ uint32_t pack_pair(float a, float b) {
  if constexpr (DT == B2_BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}
template <int DT>
__device__ __forceinline__ void unpack_pair(uint32_t w, float& lo, float& hi) {
  if constexpr (DT == B2_BF16) {
    lo = __uint_as_float(w << 16);
    hi = __uint_as_float(w & 0xffff0000u);
  } else {
    const __half2 h2 = *reinterpret_cast<const __half2*>(&w);
    lo = __low2float(h2);
    hi = __high2float(h2);
  }
}
// 32-bit word j (0 .. 15) of four 16-byte vectors
__device__ __forceinline__ uint32_t word_of(const uint4 (&v)[4], int j) {
  const uint4& u = v[j >> 2];
  return (j & 3) == 0 ? u.x : (j & 3) == 1 ? u.y : (j & 3) == 2 ? u.z : u.w;
}
template <int DT>
__device__ __forceinline__ float ld_act(const uint16_t* p) {
  return to_f32<typename dtype_of<DT>::T>(*reinterpret_cast<const typename dtype_of<DT>::T*>(p));
}
template <int DT>
__device__ __forceinline__ uint32_t splat(float v) {
  return pack_pair<DT>(v, v);
}

// 4 int8 -> 2 packed pairs (activation dtype), exact.
template <int DT>
__device__ __forceinline__ void int8x4_to_act(uint32_t w, uint32_t& lo, uint32_t& hi) {
  // bytes (0, 1) and (2, 3) of w into the low bytes of the two 16-bit halves
  const uint32_t p[2] = {prmt(w, 0u, 0x4140u), prmt(w, 0u, 0x4342u)};
  uint32_t r[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    if constexpr (DT == B2_BF16) {
      // bf16 holds 128 + m (m = the byte's low 7 bits) exactly; the byte's
      // sign bit selects 128 (w >= 0: w = m) or 256 (w < 0: w = m - 128) to
      // subtract, so the difference is the exact integer w
      r[i] = sub2<DT>(and_or(p[i], 0x007F007Fu, 0x43004300u), and_or(p[i], 0x00800080u, 0x43004300u));
    } else {
      // fp16 holds 1024 + (w + 128) exactly: (byte ^ 0x80) | 0x6400, then
      // subtract 1152
      uint32_t t;
      asm("lop3.b32 %0, %1, %2, %3, 0xBE;" : "=r"(t) : "r"(p[i]), "r"(0x00800080u), "r"(0x64006400u));
      r[i] = sub2<DT>(t, 0x64806480u);
    }
  }
  lo = r[0];
  hi = r[1];
}

// fp32 sum of 8 packed activation values.
template <int DT>
__device__ __forceinline__ float sum8(uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (DT == B2_BF16) {
      s += __uint_as_float(w[i] << 16) + __uint_as_float(w[i] & 0xFFFF0000u);
    } else {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      s += f.x + f.y;
    }
  }
  return s;
}

template <int MODE, int DT, bool ZP>
__global__ void __launch_bounds__(Cfg<MODE>::kThreads, 1)
wxa16_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const __grid_constant__ CUtensorMap tmO, const Params p) {
  using C = Cfg<MODE>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sA = smem;
  uint8_t* sB = sA + C::kStages * C::kABytesC;
  uint8_t* sP = sB + C::kBRegion;
  uint64_t* full = reinterpret_cast<uint64_t*>(sP + C::kStages * C::kPackedBytes);
  uint64_t* bready = full + C::kStages;
  uint64_t* empty = bready + C::kStages;
  uint64_t* tfull = empty + C::kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* xsready = drain + 1;  // W8 with zeros: row sums of the tile written
  uint64_t* xsfree = xsready + 2;  // ... and read by the epilogue (once per tile)
  uint64_t* bempty = xsfree + 1;   // W8: B buffer b read by its MMAs
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* xsbuf = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full) + 256);  // MODE 1 && ZP
  // 128-byte aligned (full sits on a 1024-byte boundary)
  uint8_t* sEpi = reinterpret_cast<uint8_t*>(full) + 256 + (MODE == 1 ? kXsBytes : 0);

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
      mbar_init(&xsready[a], kDequantWarps);
      mbar_init(&bempty[a], 1);
    }
    mbar_init(xsfree, 4);
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
        const int m0 = (tile % p.tiles_m) * C::BMC, n0 = (tile / p.tiles_m) * p.bn;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_or_abort(&empty[stage], phase ^ 1, p, 0xB2100001u, abort_flag)) {
            ok = false;
            break;
          }
          // the B box is bn rows (MODE 2: bn columns of 8 int32 rows)
          const uint32_t bytes = C::kABytesC + (uint32_t)p.bn * (MODE == 0 ? BK * 2 : (MODE == 1 ? BK : BK / 2));
          mbar_arrive_expect_tx(&full[stage], bytes);
          tma_load_2d(sA + stage * C::kABytesC, &tmA, kb * BK, m0, &full[stage]);
          if constexpr (MODE == 0) tma_load_2d(sB + stage * kBBytes, &tmB, kb * BK, n0, &full[stage]);
          if constexpr (MODE == 1) tma_load_2d(sP + stage * C::kPackedBytes, &tmB, kb * BK, n0, &full[stage]);
          if constexpr (MODE == 2) tma_load_2d(sP + stage * C::kPackedBytes, &tmB, n0, kb * (BK / 8), &full[stage]);
          if constexpr (MODE == 3) tma_load_2d(sP + stage * C::kPackedBytes, &tmB, kb * (BK / 2), n0, &full[stage]);
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
      const uint32_t idesc = p.idesc;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      int kbi = 0;  // k-blocks issued so far (B buffer of the W8 mode)
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
        if constexpr (C::TWO) {
          // acc half h (TMEM columns h * 256) holds rows h * 128 .. + 127;
          // each half is released separately by the epilogue of the previous tile
          const uint32_t tparity = (it & 1) ^ 1;
          for (int kb = 0; kb < kblocks; ++kb, ++kbi) {
            // B: this stage's tile, or (W8) buffer kbi & 1, filled once per use
            const int bb = C::SPLITB ? (kbi & 1) : stage;
            const uint32_t bpar = C::SPLITB ? ((kbi >> 1) & 1) : phase;
            if (!wait_or_abort(&full[stage], phase, p, 0xB2100003u, abort_flag) ||
                !wait_or_abort(&bready[bb], bpar, p, 0xB2100004u, abort_flag) ||
                (kb == 0 && !wait_or_abort(&tempty[0], tparity, p, 0xB2100002u, abort_flag))) {
              ok = false;
              break;
            }
            tc::fence_after_sync();
            const uint64_t da = tc::desc_kmajor_sw128(sA + stage * C::kABytesC);
            const uint64_t db = tc::desc_kmajor_sw128(sB + bb * kBBytes);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              tc::mma_f16_ss(tmem_base, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, (kb | k) != 0);
            if (kb == 0) {
              if (!wait_or_abort(&tempty[1], tparity, p, 0xB210000Au, abort_flag)) {
                ok = false;
                break;
              }
              tc::fence_after_sync();
            }
            // rows 128..255 of the A tile start 16 KB in (128-byte rows)
            const uint64_t da1 = tc::desc_kmajor_sw128(sA + stage * C::kABytesC + BM * BK * 2);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              tc::mma_f16_ss(tmem_base + kAccCols, da1 + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc,
                             (kb | k) != 0);
            tc::commit(&empty[stage]);
            if constexpr (C::SPLITB) tc::commit(&bempty[bb]);
            if (++stage == C::kStages) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (ok) tc::commit(&tfull[0]);
          continue;
        }
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
          const uint64_t da = tc::desc_kmajor_sw128(sA + stage * C::kABytesC);
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
    uint8_t* const stg = sEpi + q * kEpiTile;
    uint16_t* const wsz = reinterpret_cast<uint16_t*>(sEpi + kEpiBytes) + q * 2 * BN;  // MODE 1
    int it = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
      const int m0 = (tile % p.tiles_m) * C::BMC, n0 = (tile / p.tiles_m) * p.bn;
      const int acc = C::TWO ? 0 : (it & 1);
      const uint32_t acc_phase = C::TWO ? (it & 1) : ((it >> 1) & 1);
      if constexpr (MODE == 1) {
        // this tile's scales (and zeros) in shared memory, read as vectors below
        __syncwarp();  // every lane has read the previous tile's
        for (int i = lane; i < BN; i += 32) {
          const int n = n0 + i;
          const bool in = i < p.bn && n < p.N;
          wsz[i] = in ? p.scales[n] : (uint16_t)0;
          if constexpr (ZP) wsz[BN + i] = in ? p.zeros[n] : (uint16_t)0;
        }
        __syncwarp();
      }
      if (!wait_or_abort(&tfull[acc], acc_phase, p, 0xB2100005u, abort_flag)) break;
      tc::fence_after_sync();
      float xs2[2] = {0.f, 0.f};  // W8 with zeros: sum_k x[row, k] of both row halves
      if constexpr (MODE == 1 && ZP) {
        if (!wait_or_abort(&xsready[0], it & 1, p, 0xB2100008u, abort_flag)) break;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float* xb = xsbuf + h * BM + q * 32 + lane;
          xs2[h] = xb[0] + xb[2 * BM];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(xsfree);  // the dequantisers may overwrite it
      }
#pragma unroll 1
      for (int h = 0; h < (C::TWO ? 2 : 1); ++h) {
        const uint32_t tcol = C::TWO ? h * kAccCols : acc * kAccCols;
        const int row0 = m0 + h * BM + q * 32;  // first row of this warp's 32
#pragma unroll 1
        for (int c = 0; c < p.bn / 32; ++c) {
          uint32_t r[32];
          // warp-collective: every lane loads; tiles past the edge skip their
          // store, and the TMA store clips the rows / columns past M / N
          tc::tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + tcol + c * 32, r);
          tc::tmem_ld_wait();
          const int nc = n0 + c * 32;
          if (row0 >= p.M || nc >= p.N) continue;
          uint32_t packed[16];
          uint4 sv[4], zv[4];  // MODE 1: the chunk's 32 scales / zeros (16-bit pairs)
          if constexpr (MODE == 1) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              sv[j] = reinterpret_cast<const uint4*>(wsz + c * 32)[j];
              if constexpr (ZP) zv[j] = reinterpret_cast<const uint4*>(wsz + BN + c * 32)[j];
            }
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float v0 = __uint_as_float(r[2 * j]), v1 = __uint_as_float(r[2 * j + 1]);
            if constexpr (MODE == 1) {
              float s0, s1;
              unpack_pair<DT>(word_of(sv, j), s0, s1);
              if constexpr (ZP) {
                float z0, z1;
                unpack_pair<DT>(word_of(zv, j), z0, z1);
                v0 -= z0 * xs2[h];
                v1 -= z1 * xs2[h];
              }
              v0 *= s0;
              v1 *= s1;
            }
            packed[j] = pack_pair<DT>(v0, v1);
          }
          // the previous chunk's store has read the staging tile
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
          // row `lane` of the 32 x 32 tile (64 bytes, unswizzled)
          uint4* srow = reinterpret_cast<uint4*>(stg + lane * 64);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            srow[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
          tc::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmO, stg, nc, row0);
            bulk_commit();
          }
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[C::TWO ? h : acc]);
      }
    }
    // the staging tiles stay valid until the last store has completed
    if (lane == 0) bulk_wait_all();
  } else if constexpr (MODE != 0) {
    // ------------------------------ dequantisers ------------------------------
    const int d = (warp - 6) * 32 + lane;
    const int n = d & (BN - 1);  // B row (output column) this thread fills
    const int h = d / BN;        // which half of the row's 64 k
    const bool n_in = n < p.bn;  // threads past the tile width only keep the barrier counts
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    int tile_it = 0;
    int kbi = 0;  // k-blocks dequantised so far (B buffer of the W8 mode)
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++tile_it) {
      const int n0 = (tile / p.tiles_m) * p.bn;
      const bool col_ok = n_in && n0 + n < p.N;
      uint32_t s2 = 0, bz2 = 0, zr2 = 0;
      float xsum = 0.f;  // W8 with zeros: this thread's quarter of an x row
      int cur_group = -1;
      for (int kb = 0; kb < kblocks; ++kb, ++kbi) {
        if (MODE >= 2) {
          const int grp = kb * BK / p.G;
          if (grp != cur_group) {
            // GPTQ: [K/G, N]; reference layout: [N, K/G]
            const size_t gi = MODE == 2 ? (size_t)grp * p.N + n0 + n : (size_t)(n0 + n) * (p.K / p.G) + grp;
            const float sc = col_ok ? ld_act<DT>(p.scales + gi) : 0.f;
            s2 = splat<DT>(sc);
            if (ZP) {
              const float z = col_ok ? ld_act<DT>(p.zeros + gi) : 0.f;
              const float zi = fminf(fmaxf(rintf(z), -64.f), 64.f);  // bias + zi stays exact
              bz2 = splat<DT>((DT == B2_BF16 ? 128.f : 1024.f) + zi);
              zr2 = splat<DT>(-(z - zi) * sc);
            }
            cur_group = grp;
          }
        }
        const int bb = C::SPLITB ? (kbi & 1) : stage;
        if (!wait_or_abort(&full[stage], phase, p, 0xB2100006u, abort_flag) ||
            (C::SPLITB && !wait_or_abort(&bempty[bb], ((kbi >> 1) & 1) ^ 1, p, 0xB210000Bu, abort_flag))) {
          ok = false;
          break;
        }
        uint8_t* brow = sB + bb * kBBytes + n * 128;
        const int sw = n & 7;
        if (!n_in) {
        } else if constexpr (MODE == 2) {
          const uint32_t* pk = reinterpret_cast<const uint32_t*>(sP + stage * C::kPackedBytes);
#pragma unroll
          for (int rr = 0; rr < BK / 16; ++rr) {
            const int r = h * (BK / 16) + rr;
            const uint4 v = dequant8_int4<DT, ZP>(pk[r * p.bn + n], s2, bz2, zr2);
            *reinterpret_cast<uint4*>(brow + ((r ^ sw) << 4)) = v;
          }
        } else if constexpr (MODE == 3) {
          // row n of the packed tile: 32 bytes = 64 k, this thread's half is
          // one 16-byte vector; word i holds k = 32 h + 8 i .. + 7 in k order
          const uint4 pv = *reinterpret_cast<const uint4*>(sP + stage * C::kPackedBytes + n * (BK / 2) + 16 * h);
          const uint32_t wv[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 v = dequant8_int4<DT, ZP>(wv[i], s2, bz2, zr2);
            *reinterpret_cast<uint4*>(brow + (((4 * h + i) ^ sw) << 4)) = v;
          }
        } else {
          const uint4* pk = reinterpret_cast<const uint4*>(sP + stage * C::kPackedBytes + n * BK);
#pragma unroll
          for (int jj = 0; jj < BK / 32; ++jj) {
            const int j = h * (BK / 32) + jj;
            const uint4 v = pk[j];
            uint32_t o[8];
            int8x4_to_act<DT>(v.x, o[0], o[1]);
            int8x4_to_act<DT>(v.y, o[2], o[3]);
            int8x4_to_act<DT>(v.z, o[4], o[5]);
            int8x4_to_act<DT>(v.w, o[6], o[7]);
            *reinterpret_cast<uint4*>(brow + (((2 * j) ^ sw) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<uint4*>(brow + (((2 * j + 1) ^ sw) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
          }
        }
        if constexpr (MODE == 1 && ZP) {
          // row d % 256 of the x tile, k-half d / 256 (four swizzled chunks)
          const int ar = d & (2 * BM - 1), aq = d >> 8;
          const uint8_t* arow = sA + stage * C::kABytesC + ar * 128;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const uint4 v = *reinterpret_cast<const uint4*>(arow + (((4 * aq + cc) ^ (ar & 7)) << 4));
            xsum += sum8<DT>(v);
          }
          if (kb == kblocks - 1) {
            // hand the row sums to the epilogue once it has read the previous
            // tile's (xsfree completes once per tile)
            if (!wait_or_abort(xsfree, (tile_it & 1) ^ 1, p, 0xB2100009u, abort_flag)) {
              ok = false;
              break;
            }
            xsbuf[aq * 2 * BM + ar] = xsum;
            xsum = 0.f;
            __syncwarp();
            if (lane == 0) mbar_arrive(&xsready[0]);
          }
        }
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bready[bb]);
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

// Tile width for a persistent grid of `sms` CTAs: 256 or 224 columns,
// whichever finishes the tiles in less time.  A round of tiles costs one
// tile's time, and a 224-column tile measured ~97% of a 256-column one (the
// N = 224 MMA costs about as much as N = 256; the dequant work is 12.5%
// less), while narrower tiles were much slower (W4 / W8 at M = 4096,
// K = 4096: 192 columns -10..-25%, 128 columns -30..-40%).  So the model is
// rounds x (256: 100, 224: 97).  C2 (N = 14336): 7 rounds either way -> 224;
// bf16 at C2 (128-row tiles): 13 rounds of 256 against 14 of 224 -> 256;
// a two-GPU column shard (N = 7168): 4 rounds either way -> 224.
// B2_GEMM_BN overrides the choice (a multiple of 32 in 128..256; for tuning).
static int pick_bn(int tiles_m, int64_t N, int sms) {
  static const int forced = [] {
    const char* e = getenv("B2_GEMM_BN");
    const int v = e ? atoi(e) : 0;
    return (v >= 128 && v <= gemm::BN && v % 32 == 0) ? v : 0;
  }();
  if (forced) return forced;
  auto cost = [&](int bn) {
    const int64_t tiles = (int64_t)tiles_m * ((N + bn - 1) / bn);
    return ((tiles + sms - 1) / sms) * (bn == gemm::BN ? 100 : 97);
  };
  return cost(224) < cost(gemm::BN) ? 224 : gemm::BN;
}

template <int MODE, int DT, bool ZP>
static int launch_gemm(const void* x, const void* w, const void* scales, const void* zeros, void* out, int64_t M,
                       int64_t N, int64_t K, int64_t G, cudaStream_t st) {
  using namespace gemm;
  using C = Cfg<MODE>;
  if (M <= 0 || N % 8 || K % BK || (MODE >= 2 && (G % BK || K % G))) return B2_ERR_UNSUPPORTED;
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(out, 16)) return B2_ERR_UNSUPPORTED;
  unsigned* err = device_error_word();
  if (!err) {
    set_error("gemm: cannot resolve the device error word");
    return B2_ERR_LAUNCH;
  }
  const CUtensorMapDataType adt = DT == B2_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  int grid = num_sms();
  const int bn = pick_bn((int)((M + C::BMC - 1) / C::BMC), N, grid);
  CUtensorMap ta, tb, to;
  if (!make_tmap_2d(&ta, x, adt, K, M, K * 2, BK, C::BMC, CU_TENSOR_MAP_SWIZZLE_128B)) return B2_ERR_INVALID;
  bool okb;
  if (MODE == 0)
    okb = make_tmap_2d(&tb, w, adt, K, N, K * 2, BK, bn, CU_TENSOR_MAP_SWIZZLE_128B);
  else if (MODE == 1)
    okb = make_tmap_2d(&tb, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, N, K, BK, bn);
  else if (MODE == 2)
    okb = make_tmap_2d(&tb, w, CU_TENSOR_MAP_DATA_TYPE_UINT32, N, K / 8, N * 4, bn, BK / 8);
  else
    okb = make_tmap_2d(&tb, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, K / 2, N, K / 2, BK / 2, bn);
  if (!okb) return B2_ERR_INVALID;
  // output [M, N] 16-bit, stored 32 x 32 per epilogue warp
  if (!make_tmap_2d(&to, out, CU_TENSOR_MAP_DATA_TYPE_UINT16, N, M, N * 2, 32, 32)) return B2_ERR_INVALID;
  Params p;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.G = (int)G;
  p.scales = (const uint16_t*)scales;
  p.zeros = (const uint16_t*)zeros;
  p.out = (uint16_t*)out;
  p.tiles_m = (int)((M + C::BMC - 1) / C::BMC);
  p.tiles_n = (int)((N + bn - 1) / bn);
  p.bn = bn;
  p.idesc = tc::idesc_f16(BM, bn, DT == B2_BF16);
  p.err = err;
  const int ntiles = p.tiles_m * p.tiles_n;
  if (grid > ntiles) grid = ntiles;
  auto kern = wxa16_gemm_kernel<MODE, DT, ZP>;
  set_max_smem((const void*)kern, (int)C::kSmem);
  kern<<<grid, C::kThreads, C::kSmem, st>>>(ta, tb, to, p);
  return launch_status("wxa16_gemm");
}

template <int MODE>
static int launch_gemm_any(const void* x, const void* w, const void* s, const void* z, void* out, int64_t M,
                           int64_t N, int64_t K, int64_t G, int dtype, cudaStream_t st) {
  if (dtype == B2_BF16)
    return z ? launch_gemm<MODE, B2_BF16, true>(x, w, s, z, out, M, N, K, G, st)
             : launch_gemm<MODE, B2_BF16, false>(x, w, s, z, out, M, N, K, G, st);
  if (dtype == B2_F16)
    return z ? launch_gemm<MODE, B2_F16, true>(x, w, s, z, out, M, N, K, G, st)
             : launch_gemm<MODE, B2_F16, false>(x, w, s, z, out, M, N, K, G, st);
  return B2_ERR_UNSUPPORTED;
}

}  // namespace b2

using namespace b2;

// Called by b2_int4_matmul for M > 16 (fp16 / bf16, symmetric or per-group zeros).
int b2_detail_w4_gemm(const void* x, const void* w, void* out, const void* s, const void* z, int64_t M, int64_t N,
                      int64_t K, int64_t G, int dtype, cudaStream_t st) {
  return launch_gemm_any<2>(x, w, s, z, out, M, N, K, G, dtype, st);
}

// Called by b2_int4_matmul_ref for M > 16: the reference's [N, K/2] layout.
int b2_detail_w4_gemm_ref(const void* x, const void* w, void* out, const void* s, const void* z, int64_t M,
                          int64_t N, int64_t K, int64_t G, int dtype, cudaStream_t st) {
  return launch_gemm_any<3>(x, w, s, z, out, M, N, K, G, dtype, st);
}

// Called by b2_int8_matmul for M > 16 (fp16 / bf16, symmetric or per-channel zeros).
int b2_detail_w8_gemm(const void* x, const void* w, void* out, const void* s, const void* z, int64_t M, int64_t N,
                      int64_t K, int dtype, cudaStream_t st) {
  return launch_gemm_any<1>(x, w, s, z, out, M, N, K, 0, dtype, st);
}

extern "C" int b2_gemm_bf16(const void* x, const void* w, void* out, int64_t M, int64_t N, int64_t K, void* stream) {
  B2_CHECK_ARG(x && w && out, B2_ERR_INVALID, "gemm_bf16: null pointer");
  B2_CHECK_ARG(M > 0 && N > 0 && K > 0, B2_ERR_INVALID, "gemm_bf16: bad shape");
  int r = launch_gemm<0, B2_BF16, false>(x, w, nullptr, nullptr, out, M, N, K, 0, (cudaStream_t)stream);
  if (r == B2_ERR_UNSUPPORTED)
    set_error("gemm_bf16: needs N %% 8 == 0, K %% 64 == 0 and 16-byte aligned pointers");
  return r;
}

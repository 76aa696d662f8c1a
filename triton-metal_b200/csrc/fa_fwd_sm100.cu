// FlashAttention forward (sm_100a): O = softmax(scale * Q K^T [+ causal]) V
//
// Reference: flash_attention template (triton_metal/codegen/_msl_templates.py
// :1568-1767; online softmax m/l/O update at :1697-1753, causal mask
// kv_pos <= q_pos at :1610-1619, final O /= l skipped when l == 0), the
// strided Triton kernel _flash_attn_fwd (tests/test_flash_attention.py:24-104)
// and the GQA head map kv_head = q_head / n_q_per_kv (_msl_templates.py:2101).
//
// Fast path (D = 128, bf16/fp16): one CTA per pair of 128-row Q tiles of one
// (b, h), longest causal pairs first (one Q tile per CTA when the pairs would
// not fill the SMs).
//   warp 0      TMA: both Q tiles once; K tiles (3-stage ring) and V tiles
//               (2-stage) shared by the two Q tiles
//   warp 1      TMEM owner + MMA issuer: S_u = Q_u K^T (M=N=128, K=16 x 8)
//               and O_u += P_u V (P from TMEM, V the MN-major smem B operand)
//               for the two tiles in ping-pong order
//   warps 4-11  two softmax warpgroups (one per Q tile), one query row per
//               thread (TMEM lane = row): row max in the log2 domain,
//               p = exp2(s - m) (a third of them by a polynomial on the
//               FMA pipe, the rest on MUFU), row sum, P as bf16 written back into TMEM
//               over its S columns; O is rescaled in TMEM only when the
//               running max grows by more than 8 (2^8 headroom in P).
//               Final O / l -> global.
// Generic path (any D <= 256, fp32/bf16/fp16, any strides): one warp per
// query row with the same online softmax in fp32.
#include "tc_common.cuh"
#include <string.h>

namespace b2 {
namespace fa {

constexpr int BQ = 128, BKV = 128;
constexpr int kKStages = 3, kVStages = 2;
constexpr int kF16 = 0, kBF16 = 1, kTF32 = 2;  // operand formats (tcgen05 instruction descriptor codes)

// Tile geometry of the tcgen05 path for head dim HD and operand format FMT
// (kTF32: fp32 q / k / v read as tf32, fp32 output).  A tile is BQ rows of HD
// elements in 128-byte swizzle atoms; one MMA k-step is 32 bytes of K.
template <int HD_, int FMT_>
struct FaCfg {
  static constexpr int HD = HD_, FMT = FMT_;
  static constexpr int ES = FMT == kTF32 ? 4 : 2;   // element bytes
  static constexpr int KSTEP = 32 / ES;             // K elements per MMA
  static constexpr int AE = 128 / ES;               // elements per swizzle row
  static constexpr int NATOM = HD / AE;
  static constexpr int kAtom = BQ * 128;            // bytes of one atom column
  static constexpr int kTile = NATOM * kAtom;
  static constexpr size_t kSmem = (size_t)kTile * (2 + kKStages + kVStages) + 1024 + 256;
  static_assert(HD % AE == 0, "head dim must fill whole swizzle rows");
};
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.f;  // log2 units

struct Params {
  int B, Hq, Hkv, Sq, Skv, causal, q_tiles;
  int window;  // > 0 (causal only): key kv visible to qpos iff qpos - window < kv <= qpos
  int single;  // 1: one Q tile per CTA instead of a pair (small grids)
  float scale_log2;
  void* o;
  int64_t os_b, os_h, os_s;
  unsigned* err;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ bool wait_abort(uint64_t* bar, uint32_t parity, unsigned* err, unsigned code,
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
  atomicCAS(err, 0u, code);
  *abort_flag = 1;
  return false;
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 4-D tensor map coordinates: (d, s, h, b)
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int d, int s, int h, int b,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(d), "r"(s), "r"(h), "r"(b), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// Fast path v2: two Q tiles per CTA (ping-pong), P kept in TMEM.
//   TMEM (512 columns): tile u in {0, 1}: S_u / P_u at columns 256u, O_u at
//   256u + 128.  P_u (bf16, two per 32-bit column) overwrites the first 64
//   columns of S_u and is read by the TMEM-A form of tcgen05.mma.
//   MMA issue order per KV block j:  PV_0(j), S_0(j+1), PV_1(j), S_1(j+1),
//   so the tensor core works on one tile while the other tile's softmax
//   warpgroup runs.  MMAs from the single issuing thread execute in order,
//   which orders S_u(j+1) after PV_u(j) (both use the S/P columns) and makes
//   O_u quiescent whenever S_u(j) is complete.
//   warps: 0 TMA, 1 TMEM owner + MMA issuer, 4-7 softmax tile 0,
//          8-11 softmax tile 1 (warp w reads TMEM lanes 32 (w % 4) ..).
// ---------------------------------------------------------------------------
constexpr int kThreads2 = 384;

// D[tmem] (+)= A[tmem] * B[smem]; kind::f16 or kind::tf32 by FMT
template <int FMT>
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  if constexpr (FMT == kTF32) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}
// D[tmem] (+)= A[smem] * B[smem]^T; kind::f16 or kind::tf32 by FMT
template <int FMT>
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  if constexpr (FMT == kTF32) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    tc::mma_f16_ss(d_tmem, a_desc, b_desc, idesc, accumulate);
  }
}
// instruction descriptor: fp32 accumulate, A / B format FMT (0 f16, 1 bf16, 2 tf32)
__host__ __device__ constexpr uint32_t idesc_fmt(int M, int N, int fmt, bool b_mn_major) {
  return (1u << 4) | ((uint32_t)fmt << 7) | ((uint32_t)fmt << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// Paired fp32 arithmetic of sm_100 (one instruction for two lanes of a
// 64-bit register pair) and the 3-input max: the softmax warps issue one
// instruction per two scores for the scale, the row sum and the max.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  return (uint64_t)__float_as_uint(a) | ((uint64_t)__float_as_uint(b) << 32);
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t fma_f2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add_f2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// exp2 of two lanes on the FMA pipe, to take part of the softmax's
// exponentials off the MUFU unit (the method of FlashAttention-4: Cody-Waite
// split x = j + f, j = rint(x), |f| <= 1/2, then a polynomial for 2^f and j
// added into the exponent field).  The cubic is this file's own relative
// minimax fit of 2^f on [-1/2, 1/2] (max relative error 7.5e-5, below the
// 2^-9 / 2^-12 rounding of the 16-bit P it feeds).  x <= 8 here; x is clamped
// at -125 so that 2^j stays a normal number.
__device__ __forceinline__ uint64_t exp2_poly_f2(uint64_t x2) {
  const uint64_t x = f2_pack(fmaxf(f2_lo(x2), -125.f), fmaxf(f2_hi(x2), -125.f));
  const float kRound = 12582912.f;  // 1.5 * 2^23: x + kRound rounds x to an integer in the low mantissa bits
  const uint64_t t = add_f2(x, f2_pack(kRound, kRound));
  const uint64_t j = add_f2(t, f2_pack(-kRound, -kRound));
  const uint64_t fr = fma_f2(j, f2_pack(-1.f, -1.f), x);
  uint64_t q = fma_f2(f2_pack(0.05517132f, 0.05517132f), fr, f2_pack(0.24261054f, 0.24261054f));
  q = fma_f2(q, fr, f2_pack(0.69326097f, 0.69326097f));
  q = fma_f2(q, fr, f2_pack(0.99992812f, 0.99992812f));
  // bits(t) = 0x4B400000 + j, so bits(t) << 23 = j << 23 (mod 2^32)
  const uint32_t lo = (uint32_t)t * (1u << 23) + (uint32_t)q;
  const uint32_t hi = (uint32_t)(t >> 32) * (1u << 23) + (uint32_t)(q >> 32);
  return (uint64_t)lo | ((uint64_t)hi << 32);
}

__device__ __forceinline__ bool key_masked(int kv, int qpos, const Params& p) {
  return kv >= p.Skv || (p.causal && kv > qpos) || (p.window > 0 && kv <= qpos - p.window);
}

// Row max of the raw S row (this thread's TMEM lane), masked keys -> -inf.
template <bool MASK>
__device__ __forceinline__ float row_max(uint32_t tS, int kv0, int qpos, const Params& p) {
  float mx = -INFINITY;
  // two 32-column loads per wait: 64 columns in flight
#pragma unroll 1
  for (int c = 0; c < 4; c += 2) {
    uint32_t sv[64];
    tc::tmem_ld_32x32b_x32(tS + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(sv));
    tc::tmem_ld_32x32b_x32(tS + 32 * c + 32, *reinterpret_cast<uint32_t(*)[32]>(sv + 32));
    tc::tmem_ld_wait();
#pragma unroll
    for (int e = 0; e < 64; e += 2) {
      float v0 = __uint_as_float(sv[e]), v1 = __uint_as_float(sv[e + 1]);
      if constexpr (MASK) {
        const int kv = kv0 + 32 * c + e;
        if (key_masked(kv, qpos, p)) v0 = -INFINITY;
        if (key_masked(kv + 1, qpos, p)) v1 = -INFINITY;
      }
      mx = max3(mx, v0, v1);
    }
  }
  return mx;
}

// p = exp2(s * scale_log2 - m) written over the S columns (P for the TMEM-A
// MMA): 16-bit pairs, or fp32 for the tf32 path; returns the row sum of p
// (two partial sums, even and odd keys, in one register pair).
template <bool MASK, int FMT>
__device__ __forceinline__ float exp_to_p(uint32_t tS, int kv0, int qpos, float mref, const Params& p) {
  uint64_t rs = 0;
  const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2), nm2 = f2_pack(-mref, -mref);
#pragma unroll 1
  for (int c = 0; c < 4; c += 2) {
    uint32_t sv[64];
    tc::tmem_ld_32x32b_x32(tS + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(sv));
    tc::tmem_ld_32x32b_x32(tS + 32 * c + 32, *reinterpret_cast<uint32_t(*)[32]>(sv + 32));
    tc::tmem_ld_wait();
    uint32_t pk[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const uint64_t x = fma_f2((uint64_t)sv[2 * e] | ((uint64_t)sv[2 * e + 1] << 32), sc2, nm2);
      float p0, p1;
      // ~1/3 of the pairs on the FMA pipe (measured at C3: 1/4 and 1/3 both
      // ~1020 TF/s, 3/8 ~1005, 1/2 ~965; all-MUFU ~970)
      if (FMT != kTF32 && e % 3 == 2) {
        const uint64_t y = exp2_poly_f2(x);
        p0 = f2_lo(y);
        p1 = f2_hi(y);
      } else {
        p0 = ex2(f2_lo(x));
        p1 = ex2(f2_hi(x));
      }
      if constexpr (MASK) {
        const int kv = kv0 + 32 * c + 2 * e;
        if (key_masked(kv, qpos, p)) p0 = 0.f;
        if (key_masked(kv + 1, qpos, p)) p1 = 0.f;
      }
      rs = add_f2(rs, f2_pack(p0, p1));
      if constexpr (FMT == kF16) {
        __half2 hv = __floats2half2_rn(p0, p1);
        pk[e] = *reinterpret_cast<uint32_t*>(&hv);
      } else if constexpr (FMT == kBF16) {
        __nv_bfloat162 hv = __floats2bfloat162_rn(p0, p1);
        pk[e] = *reinterpret_cast<uint32_t*>(&hv);
      } else {
        sv[2 * e] = __float_as_uint(p0);
        sv[2 * e + 1] = __float_as_uint(p1);
      }
    }
    if constexpr (FMT == kTF32) {
      tmem_st_32x32b_x32(tS + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(sv));
      tmem_st_32x32b_x32(tS + 32 * c + 32, *reinterpret_cast<uint32_t(*)[32]>(sv + 32));
    } else {
      tmem_st_32x32b_x32(tS + 16 * c, pk);
    }
  }
  return f2_lo(rs) + f2_hi(rs);
}

template <int HD, int FMT>
__global__ void __launch_bounds__(kThreads2, 1)
fa_fwd2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, const Params p) {
  using Cf = FaCfg<HD, FMT>;
  constexpr int kTile = Cf::kTile, kAtom = Cf::kAtom;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQ = smem;                      // 2 tiles
  uint8_t* sK = sQ + 2 * kTile;
  uint8_t* sV = sK + kKStages * kTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kVStages * kTile);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + kKStages;
  uint64_t* v_full = k_empty + kKStages;
  uint64_t* v_empty = v_full + kVStages;
  uint64_t* s_full = v_empty + kVStages;  // [2] per tile
  uint64_t* p_ready = s_full + 2;         // [2]
  uint64_t* o_done = p_ready + 2;         // [2]
  uint64_t* drain = o_done + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // one unit = a pair of Q tiles, or one Q tile when the grid would not fill
  // the SMs (p.single: the second softmax warpgroup idles, the CTAs halve)
  const int per = p.single ? 1 : 2;
  const int nunits = (p.q_tiles + per - 1) / per;
  const int pi = nunits - 1 - (int)blockIdx.x;  // longest causal units first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Hq / p.Hkv);
  const int nkv_all = (p.Skv + BKV - 1) / BKV;
  // Tile u visits KV tiles kb[u] .. nkv[u]-1 (kb > 0 only with a sliding
  // window); the pair shares the K/V ring over the union jb .. nkv_max-1.
  int q0[2], nkv[2], kb[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    q0[u] = (per * pi + u) * BQ;
    nkv[u] = (u < per && per * pi + u < p.q_tiles)
                 ? (p.causal ? min(nkv_all, (q0[u] + BQ - 1) / BKV + 1) : nkv_all)
                 : 0;
    kb[u] = p.window > 0 ? min(max(0, q0[u] - p.window + 1) / BKV, nkv[u]) : 0;
  }
  const int nkv_max = max(nkv[0], nkv[1]);
  const int jb = kb[0];
  auto active = [&](int u, int j) { return j >= kb[u] && j < nkv[u]; };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < kVStages; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int u = 0; u < 2; ++u) {
      mbar_init(&s_full[u], 1);
      mbar_init(&p_ready[u], 4);
      mbar_init(&o_done[u], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_holder, 512);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ---------------------------------- TMA ----------------------------------
    if (lane == 0) {
      const int ntiles = nkv[1] > 0 ? 2 : 1;
      mbar_arrive_expect_tx(q_full, ntiles * kTile);
      for (int u = 0; u < ntiles; ++u)
#pragma unroll
        for (int a = 0; a < Cf::NATOM; ++a) tma_load_4d(sQ + u * kTile + a * kAtom, &tmQ, a * Cf::AE, q0[u], h, b, q_full);
      int kst = 0, vst = 0;
      uint32_t kph = 0, vph = 0;
      for (int j = jb; j < nkv_max; ++j) {
        if (!wait_abort(&k_empty[kst], kph ^ 1, p.err, 0xB2300001u, abort_flag)) break;
        mbar_arrive_expect_tx(&k_full[kst], kTile);
#pragma unroll
        for (int a = 0; a < Cf::NATOM; ++a)
          tma_load_4d(sK + kst * kTile + a * kAtom, &tmK, a * Cf::AE, j * BKV, hk, b, &k_full[kst]);
        if (!wait_abort(&v_empty[vst], vph ^ 1, p.err, 0xB2300002u, abort_flag)) break;
        mbar_arrive_expect_tx(&v_full[vst], kTile);
#pragma unroll
        for (int a = 0; a < Cf::NATOM; ++a)
          tma_load_4d(sV + vst * kTile + a * kAtom, &tmV, a * Cf::AE, j * BKV, hk, b, &v_full[vst]);
        if (++kst == kKStages) { kst = 0; kph ^= 1; }
        if (++vst == kVStages) { vst = 0; vph ^= 1; }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------- MMA ----------------------------------
    if (lane == 0) {
      constexpr uint32_t idS = idesc_fmt(BQ, BKV, FMT, false);
      constexpr uint32_t idPV = idesc_fmt(BQ, HD, FMT, true);
      bool ok = wait_abort(q_full, 0, p.err, 0xB2300003u, abort_flag);
      int kst = 0, vst = 0;
      uint32_t kph = 0, vph = 0;
      auto issue_s = [&](int u) {
#pragma unroll
        for (int kk = 0; kk < HD / Cf::KSTEP; ++kk) {
          const uint64_t da = tc::desc_kmajor_sw128(sQ + u * kTile + (kk >> 2) * kAtom + (kk & 3) * 32);
          const uint64_t db = tc::desc_kmajor_sw128(sK + kst * kTile + (kk >> 2) * kAtom + (kk & 3) * 32);
          mma_ss<FMT>(tmem + 256 * u, da, db, idS, kk != 0);
        }
        tc::commit(&s_full[u]);
      };
      // prologue: S_u(0)
      if (ok && nkv_max > jb) {
        ok = wait_abort(&k_full[kst], kph, p.err, 0xB2300004u, abort_flag);
        if (ok) {
          tc::fence_after_sync();
          for (int u = 0; u < 2; ++u)
            if (active(u, jb)) issue_s(u);
          tc::commit(&k_empty[kst]);
          if (++kst == kKStages) { kst = 0; kph ^= 1; }
        }
      }
      for (int j = jb; j < nkv_max && ok; ++j) {
        if (!wait_abort(&v_full[vst], vph, p.err, 0xB2300005u, abort_flag)) {
          ok = false;
          break;
        }
        const bool next_k = active(0, j + 1) || active(1, j + 1);
        bool k_waited = false;
        for (int u = 0; u < 2 && ok; ++u) {
          if (active(u, j)) {
            if (!wait_abort(&p_ready[u], (j - kb[u]) & 1, p.err, 0xB2300006u, abort_flag)) {
              ok = false;
              break;
            }
            tc::fence_after_sync();
#pragma unroll
            // one k-step = KSTEP keys: KSTEP rows of V, 8 TMEM columns of P.
            // V is the MN-major B operand: 128-byte rows along d, atoms of
            // 8 rows (16-bit, 128B swizzle) or of 4 rows (tf32, 128B swizzle
            // with 32-byte atomicity, descriptor layout 1) stacked along K.
            for (int kk = 0; kk < BKV / Cf::KSTEP; ++kk) {
              const uint64_t db =
                  FMT == kTF32 ? tc::smem_desc(sV + vst * kTile + kk * Cf::KSTEP * 128, kAtom, 512, 1)
                               : tc::smem_desc(sV + vst * kTile + kk * Cf::KSTEP * 128, kAtom, 1024, tc::kSwizzle128B);
              mma_ts<FMT>(tmem + 256 * u + 128, tmem + 256 * u + kk * 8, db, idPV, (j != kb[u]) || kk != 0);
            }
            if (j == nkv[u] - 1) tc::commit(&o_done[u]);
          }
          if (active(u, j + 1)) {
            if (!k_waited) {
              if (!wait_abort(&k_full[kst], kph, p.err, 0xB2300007u, abort_flag)) {
                ok = false;
                break;
              }
              tc::fence_after_sync();
              k_waited = true;
            }
            issue_s(u);
          }
        }
        if (!ok) break;
        tc::commit(&v_empty[vst]);
        if (++vst == kVStages) { vst = 0; vph ^= 1; }
        if (next_k) {
          tc::commit(&k_empty[kst]);
          if (++kst == kKStages) { kst = 0; kph ^= 1; }
        }
      }
      if (!ok) {
        tc::commit(drain);
        mbar_wait(drain, 0, p.err, 0xB2300008u);
      }
    }
  } else if (warp >= 4) {
    // -------------------------------- softmax --------------------------------
    const int u = (warp - 4) >> 2;
    const int qw = warp & 3;
    const int r = qw * 32 + lane;
    const int qpos = q0[u] + r;
    const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
    const uint32_t tS = tmem + 256 * u + lane_off, tO = tS + 128;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = kb[u]; j < nkv[u] && ok; ++j) {
      if (!wait_abort(&s_full[u], (j - kb[u]) & 1, p.err, 0xB2300009u, abort_flag)) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const int kv0 = j * BKV;
      const bool need_mask = (p.causal && kv0 + BKV - 1 > q0[u]) || kv0 + BKV > p.Skv ||
                             (p.window > 0 && kv0 <= q0[u] + BQ - 1 - p.window);
      // pass 1: row max of the raw scores (scale > 0 commutes with max)
      float mx = need_mask ? row_max<true>(tS, kv0, qpos, p) : row_max<false>(tS, kv0, qpos, p);
      mx *= p.scale_log2;
      // lazy, warp-uniform rescale of O (O_u is quiescent: PV_u(j-1) finished)
      const bool need = mx > m_used + kRescaleThreshold;
      const float alpha = need ? ((m_used == -INFINITY) ? 0.f : ex2(m_used - mx)) : 1.f;
      if (need) {
        l *= alpha;
        m_used = mx;
      }
      if (__any_sync(0xffffffffu, need) && j > kb[u]) {
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tc::tmem_ld_32x32b_x32(tO + 32 * c, o);
          tc::tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st_32x32b_x32(tO + 32 * c, o);
        }
      }
      // pass 2: p = exp2(s * scale - m) -> bf16 pairs over the S columns already read
      const float mref = (m_used == -INFINITY) ? 0.f : m_used;
      const float rs = need_mask ? exp_to_p<true, FMT>(tS, kv0, qpos, mref, p)
                                 : exp_to_p<false, FMT>(tS, kv0, qpos, mref, p);
      l += rs;
      tmem_st_wait();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[u]);
    }
    // epilogue: O_u / l -> global (rows beyond Sq are not stored)
    if (ok && nkv[u] > kb[u] && wait_abort(&o_done[u], 0, p.err, 0xB230000Au, abort_flag)) {
      tc::fence_after_sync();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int64_t orow = b * p.os_b + h * p.os_h + (int64_t)qpos * p.os_s;
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t o[32];
        tc::tmem_ld_32x32b_x32(tO + 32 * c, o);
        tc::tmem_ld_wait();
        if (qpos < p.Sq) {
          if constexpr (FMT == kTF32) {
            float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.o) + orow + 32 * c);
#pragma unroll
            for (int e = 0; e < 8; ++e)
              dst[e] = make_float4(__uint_as_float(o[4 * e]) * inv, __uint_as_float(o[4 * e + 1]) * inv,
                                   __uint_as_float(o[4 * e + 2]) * inv, __uint_as_float(o[4 * e + 3]) * inv);
          } else {
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const float a = __uint_as_float(o[2 * e]) * inv, bb = __uint_as_float(o[2 * e + 1]) * inv;
              if constexpr (FMT == kF16) {
                __half2 hv = __floats2half2_rn(a, bb);
                pk[e] = *reinterpret_cast<uint32_t*>(&hv);
              } else {
                __nv_bfloat162 hv = __floats2bfloat162_rn(a, bb);
                pk[e] = *reinterpret_cast<uint32_t*>(&hv);
              }
            }
            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.o) + orow + 32 * c);
#pragma unroll
            for (int e = 0; e < 4; ++e) dst[e] = make_uint4(pk[4 * e], pk[4 * e + 1], pk[4 * e + 2], pk[4 * e + 3]);
          }
        }
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, 512);
  }
}


// ---------------------------------------------------------------------------
// Generic path: one warp per query row, fp32 online softmax (same update as
// the reference template, _msl_templates.py:1712-1743).  Any D <= 256.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float ldf(const T* p) {
  if constexpr (sizeof(T) == 4) return *reinterpret_cast<const float*>(p);
  else return to_f32<T>(*p);
}
template <typename T>
__device__ __forceinline__ void stf(T* p, float v) {
  if constexpr (sizeof(T) == 4) *reinterpret_cast<float*>(p) = v;
  else *p = from_f32<T>(v);
}

struct GenParams {
  const void *q, *k, *v;
  void* o;
  int B, Hq, Hkv, Sq, Skv, D, causal;
  int window;  // > 0 (causal only): keys s - window + 1 .. s (sliding window)
  float scale;
  int64_t qs[3], ks[3], vs[3], os[3];
};

template <typename T>
__global__ void __launch_bounds__(128) fa_generic_kernel(const GenParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 4 + warp;
  if (row >= (int64_t)p.B * p.Hq * p.Sq) return;
  const int s = row % p.Sq;
  const int h = (row / p.Sq) % p.Hq;
  const int b = row / ((int64_t)p.Sq * p.Hq);
  const int hk = h / (p.Hq / p.Hkv);
  const T* q = (const T*)p.q + b * p.qs[0] + h * p.qs[1] + (int64_t)s * p.qs[2];
  const T* kb = (const T*)p.k + b * p.ks[0] + hk * p.ks[1];
  const T* vb = (const T*)p.v + b * p.vs[0] + hk * p.vs[1];
  constexpr int MAXE = 8;
  float qv[MAXE], acc[MAXE];
#pragma unroll
  for (int e = 0; e < MAXE; ++e) {
    const int d = lane + 32 * e;
    qv[e] = d < p.D ? ldf(q + d) * p.scale : 0.f;
    acc[e] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const int kend = p.causal ? min(p.Skv, s + 1) : p.Skv;
  const int kbeg = p.window > 0 ? max(0, s - p.window + 1) : 0;
  for (int j = kbeg; j < kend; ++j) {
    const T* kr = kb + (int64_t)j * p.ks[2];
    float dot = 0.f;
#pragma unroll
    for (int e = 0; e < MAXE; ++e) {
      const int d = lane + 32 * e;
      if (d < p.D) dot += qv[e] * ldf(kr + d);
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    const float mn = fmaxf(m, dot);
    const float alpha = __expf(m - mn), pj = __expf(dot - mn);
    l = l * alpha + pj;
    const T* vr = vb + (int64_t)j * p.vs[2];
#pragma unroll
    for (int e = 0; e < MAXE; ++e) {
      const int d = lane + 32 * e;
      acc[e] = acc[e] * alpha + (d < p.D ? pj * ldf(vr + d) : 0.f);
    }
    m = mn;
  }
  T* o = (T*)p.o + b * p.os[0] + h * p.os[1] + (int64_t)s * p.os[2];
  const float inv = l > 0.f ? 1.f / l : 0.f;  // all-masked row -> 0 (reference nan_to_num)
#pragma unroll
  for (int e = 0; e < MAXE; ++e) {
    const int d = lane + 32 * e;
    if (d < p.D) stf(o + d, acc[e] * inv);
  }
}

}  // namespace fa

// dims (d, s, h, b), element strides (b, h, s); box = one swizzle row
// (box_d elements = 128 bytes) x 128 rows.
// mn_major_tf32: the 128-byte swizzle with 32-byte atomicity that the MMA's
// MN-major tf32 operand layout (SWIZZLE_128B_BASE32B) expects (V of the tf32 path).
static bool make_tmap_4d(CUtensorMap* map, const void* base, int dtype, int64_t D, int64_t S, int64_t H, int64_t B,
                         const int64_t* strides_elems, bool mn_major_tf32 = false) {
  // dims (d, s, h, b); strides in bytes for s, h, b
  typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                               const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                               CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return false;
    fn = reinterpret_cast<EncodeFn>(p);
  }
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  const cuuint64_t es = dtype == B2_F32 ? 4 : 2;
  const cuuint64_t strides[3] = {(cuuint64_t)strides_elems[2] * es, (cuuint64_t)strides_elems[1] * es,
                                 (cuuint64_t)strides_elems[0] * es};
  const cuuint32_t box[4] = {(cuuint32_t)(128 / es), 128, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt = dtype == B2_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == B2_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  return fn(map, dt, 4, const_cast<void*>(base),
            dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            mn_major_tf32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// element strides whose byte values are multiples of 16 (TMA)
static bool strides_ok(const int64_t* s, int dtype) {
  const int64_t m = dtype == B2_F32 ? 4 : 8;
  return s[0] % m == 0 && s[1] % m == 0 && s[2] % m == 0;
}

template <int HD, int FMT>
static void launch_fa_tc(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const fa::Params& p,
                         dim3 grid, cudaStream_t st) {
  using Cf = fa::FaCfg<HD, FMT>;
  set_max_smem((const void*)fa::fa_fwd2_kernel<HD, FMT>, (int)Cf::kSmem);
  fa::fa_fwd2_kernel<HD, FMT><<<grid, fa::kThreads2, Cf::kSmem, st>>>(tq, tk, tv, p);
}

}  // namespace b2

using namespace b2;

static int launch_fa_generic(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t Hq,
                             int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D, const int64_t* qs, const int64_t* ks,
                             const int64_t* vs, const int64_t* os, float scale, int causal, int window, int dtype,
                             cudaStream_t st) {
  fa::GenParams g;
  g.q = q;
  g.k = k;
  g.v = v;
  g.o = o;
  g.B = (int)B;
  g.Hq = (int)Hq;
  g.Hkv = (int)Hkv;
  g.Sq = (int)Sq;
  g.Skv = (int)Skv;
  g.D = (int)D;
  g.causal = causal;
  g.window = window;
  g.scale = scale;
  for (int i = 0; i < 3; ++i) {
    g.qs[i] = qs[i];
    g.ks[i] = ks[i];
    g.vs[i] = vs[i];
    g.os[i] = os[i];
  }
  const int64_t rows = B * Hq * Sq;
  const unsigned blocks = (unsigned)((rows + 3) / 4);
  if (dtype == B2_F32) fa::fa_generic_kernel<float><<<blocks, 128, 0, st>>>(g);
  else if (dtype == B2_BF16) fa::fa_generic_kernel<__nv_bfloat16><<<blocks, 128, 0, st>>>(g);
  else fa::fa_generic_kernel<__half><<<blocks, 128, 0, st>>>(g);
  return launch_status("fa_generic");
}

static int fa_fwd_impl(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t Hq, int64_t Hkv,
                       int64_t Sq, int64_t Skv, int64_t D, const int64_t* qs, const int64_t* ks, const int64_t* vs,
                       const int64_t* os, float scale, int causal, int window, int dtype, void* stream) {
  B2_CHECK_ARG(q && k && v && o && qs && ks && vs && os, B2_ERR_INVALID, "flash_attn_fwd: null pointer");
  B2_CHECK_ARG(B > 0 && Hq > 0 && Hkv > 0 && Sq >= 0 && Skv >= 0 && D > 0, B2_ERR_INVALID,
               "flash_attn_fwd: bad shape");
  B2_CHECK_ARG(Hq % Hkv == 0, B2_ERR_INVALID, "flash_attn_fwd: Hq=%lld not a multiple of Hkv=%lld", (long long)Hq,
               (long long)Hkv);
  B2_CHECK_ARG(!causal || Sq == Skv, B2_ERR_INVALID, "flash_attn_fwd: causal needs Sq == Skv (square tril mask)");
  B2_CHECK_ARG(dtype == B2_F16 || dtype == B2_BF16 || dtype == B2_F32, B2_ERR_DTYPE, "flash_attn_fwd: dtype %d",
               dtype);
  B2_CHECK_ARG(D <= 256, B2_ERR_UNSUPPORTED, "flash_attn_fwd: D=%lld > 256", (long long)D);
  if (Sq == 0) return B2_OK;
  cudaStream_t st = (cudaStream_t)stream;
  // tcgen05 path: D = 128 with 16-bit operands, D = 64 with 16-bit operands or
  // fp32 (read as tf32, fp32 output); TMA-able strides and base addresses
  const bool shape_ok = (D == 128 && dtype != B2_F32) || D == 64;
  const bool fast = shape_ok && Skv > 0 && strides_ok(qs, dtype) && strides_ok(ks, dtype) && strides_ok(vs, dtype) &&
                    strides_ok(os, dtype) && aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(o, 16) &&
                    B <= 65535 && Hq <= 65535;
  if (fast) {
    unsigned* err = device_error_word();
    CUtensorMap tq, tk, tv;
    if (err && make_tmap_4d(&tq, q, dtype, D, Sq, Hq, B, qs) && make_tmap_4d(&tk, k, dtype, D, Skv, Hkv, B, ks) &&
        make_tmap_4d(&tv, v, dtype, D, Skv, Hkv, B, vs, dtype == B2_F32)) {
      fa::Params p;
      p.B = (int)B;
      p.Hq = (int)Hq;
      p.Hkv = (int)Hkv;
      p.Sq = (int)Sq;
      p.Skv = (int)Skv;
      p.causal = causal;
      p.window = window;
      p.q_tiles = (int)((Sq + fa::BQ - 1) / fa::BQ);
      p.scale_log2 = scale * fa::kLog2e;
      p.o = o;
      p.os_b = os[0];
      p.os_h = os[1];
      p.os_s = os[2];
      p.err = err;
      // Q-tile pairs, or single Q tiles when the pairs would not fill the SMs
      p.single = (int64_t)((p.q_tiles + 1) / 2) * Hq * B < num_sms() ? 1 : 0;
      dim3 grid(p.single ? p.q_tiles : (p.q_tiles + 1) / 2, (unsigned)Hq, (unsigned)B);
      if (D == 128) {
        if (dtype == B2_F16) launch_fa_tc<128, fa::kF16>(tq, tk, tv, p, grid, st);
        else launch_fa_tc<128, fa::kBF16>(tq, tk, tv, p, grid, st);
      } else {
        if (dtype == B2_F16) launch_fa_tc<64, fa::kF16>(tq, tk, tv, p, grid, st);
        else if (dtype == B2_BF16) launch_fa_tc<64, fa::kBF16>(tq, tk, tv, p, grid, st);
        else launch_fa_tc<64, fa::kTF32>(tq, tk, tv, p, grid, st);
      }
      return launch_status("fa_fwd");
    }
  }
  return launch_fa_generic(q, k, v, o, B, Hq, Hkv, Sq, Skv, D, qs, ks, vs, os, scale, causal, window, dtype, st);
}

extern "C" int b2_flash_attn_fwd(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t Hq,
                                 int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D, const int64_t* qs,
                                 const int64_t* ks, const int64_t* vs, const int64_t* os, float scale, int causal,
                                 int dtype, void* stream) {
  return fa_fwd_impl(q, k, v, o, B, Hq, Hkv, Sq, Skv, D, qs, ks, vs, os, scale, causal, 0, dtype, stream);
}

// Causal sliding-window FlashAttention (Mistral-style): query s attends to
// keys s - window + 1 .. s.  The prefill counterpart of the decode window
// (sliding_window_attention, _msl_templates.py:3335-3431).  Same dispatch as
// b2_flash_attn_fwd: the tcgen05 kernel for D = 128 bf16/fp16 (each Q tile
// visits only the KV tiles its window reaches), else the CUDA-core kernel.
extern "C" int b2_flash_attn_fwd_window(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t Hq,
                                        int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D, const int64_t* qs,
                                        const int64_t* ks, const int64_t* vs, const int64_t* os, float scale,
                                        int64_t window, int dtype, void* stream) {
  B2_CHECK_ARG(window > 0 && window <= 2147483647, B2_ERR_INVALID, "flash_attn_fwd_window: window must be > 0");
  return fa_fwd_impl(q, k, v, o, B, Hq, Hkv, Sq, Skv, D, qs, ks, vs, os, scale, 1, (int)window, dtype, stream);
}

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
// Kernel B (one CTA per (b, h, 64 columns of Dv)) carries the fp32 state
// through the chunks in order on fp16 tensor cores (columns of the state are
// independent: the transition acts on the Dk side only) and forms each
// chunk's outputs in the same pass, so neither V' nor the per-chunk state
// ever leaves the SM.
#include "b2_common.cuh"
#include "tc_common.cuh"
#include <string.h>
#include <type_traits>

namespace b2 {
namespace kda {

constexpr int C = 64, DK = 128, DV = 128;

// Workspace block per (b, h, chunk), laid out as kernel B's shared-memory
// stages so that bulk copies move it: fp16 W and K e^{G_last - G} [64][136]
// (rows padded by 8 halves: ldmatrix rows on distinct banks), fp32
// e^{G_last} [128] (the state CTA's part), fp16 scale Q e^G [64][136] and
// A_qk [64][72] (the output CTA's part), then fp16 U for state columns 0-63
// and 64-127 as two [64][72] tiles.  80,384 bytes.  The fp16 tiles only feed
// 10-bit-mantissa MMA operands and are O(1); the state itself is carried in
// fp32 registers.
constexpr int LR = DK + 8;    // halves: W, Kr, Qg rows
constexpr int LA = C + 8;     // halves: A_qk rows
constexpr int LUS = 64 + 8;   // halves: rows of one 64-column U tile
constexpr uint32_t kBW = 0;
constexpr uint32_t kBKr = kBW + C * LR * 2;
constexpr uint32_t kBGl = kBKr + C * LR * 2;
constexpr uint32_t kBQg = kBGl + DK * 4;
constexpr uint32_t kBAq = kBQg + C * LR * 2;
constexpr uint32_t kBShared = kBAq + C * LA * 2;  // bytes shared by the head's CTAs
constexpr uint32_t kBUTile = C * LUS * 2;          // one U tile
constexpr uint32_t kBU = kBShared;                 // U tile h at kBU + h * kBUTile
constexpr uint32_t kWsBlockBytes = kBU + 2 * kBUTile;
constexpr size_t kWsBlock = kWsBlockBytes / 4;     // floats
constexpr uint32_t kBStatePart = kBQg;             // [0, kBQg): W, Kr, e^{G_last}
constexpr uint32_t kBOutPart = kBShared - kBQg;    // [kBQg, kBShared): Qg, A_qk
static_assert(kBQg % 16 == 0 && kBShared % 16 == 0 && kBUTile % 16 == 0, "bulk copy sizes");
__device__ __forceinline__ __half* ws_h(float* blk, uint32_t byte_off) {
  return reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(blk) + byte_off);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ---------------------------------------------------------------------------
// Kernel A: intra-chunk WY/UT transform on the 5th-gen tensor cores, one CTA
// per (b, h, chunk), 256 threads, two CTAs per SM.  Thread (dp, I) owns the
// column pair d = 2 dp, 2 dp + 1 of the 16 rows of block I (rows 16 I ..).
//  1. G = in-chunk cumsum of g: block prefix in registers, block offsets and
//     the reference rows (each block's first row, the last row) via smem.
//  2. Every exponential is split at a per-block reference row r0 = 16 I so
//     that each bf16 factor stays in range (G is non-increasing along t):
//        i side  L_i  = k_i e^{G_i - G_r0(I(i))}                 (<= 1)
//                Lq_i = scale q_i e^{G_i - G_r0(I(i))}           (<= 1)
//        j side  K^(I')_j = k_j e^{G_r0(I') - G_j},  j < 16 (I' + 1)
//     (<= 1 for j in an earlier block, up to e^{gap} inside block I', gap =
//     max_d (G_r0 - G_next r0)), so that for i in block I' and j <= i
//        A_kk[i][j] = beta_i L_i . K^(I')_j,   A_qk[i][j] = Lq_i . K^(I')_j.
//     Blocks with gap > 80 (beyond bf16 / fp32 range of the factors) get
//     their diagonal 16 x 16 block recomputed exactly on CUDA cores.
//  3. Two tcgen05.mma (bf16 operands, K = 128, M = N = 128): A = the j-side
//     rows of block rows 3 and 2 (then 1 and 0), B = [L; Lq] for all 64 i;
//     every lower block of A_kk and A_qk lands in TMEM.
//  4. T = (I + A_kk)^-1: diagonal 16 x 16 blocks by column substitution
//     (fp32), then the off-diagonal blocks in two levels of the 2 x 2 block
//     inverse T_BA = -T_BB A_BA T_AA (16- then 32-row halves) on tf32 MMAs.
//  5. W^T = (beta K e^G)^T T^T and U^T = (beta V)^T T^T as two tcgen05.mma
//     (bf16: v arrives by TMA as the MN-major A operand and beta is folded
//     into the columns of T)
//     (M = 128 = Dk / Dv, N = 64, K = 64), bf16 operands, fp32 in TMEM.
//  6. W, U, A_qk, scale Q e^G, K e^{G_last - G} (fp16) and e^{G_last} go to
//     the workspace block of this chunk in kernel B's stage layout.
// ---------------------------------------------------------------------------
namespace prep {
constexpr int kThreads = 256;
constexpr int LT = C + 4;  // fp32 row stride of A_kk / A_qk / T scratch
// region R: A_kk MMA operands (bf16, K-major, 128-byte swizzle, 1024-aligned);
// K-blocks of 64 elements each hold `rows` rows
constexpr uint32_t kRowsAA = 112;                        // j side of block rows 3 (64) and 2 (48)
constexpr uint32_t kRowsAB = 48;                         // j side of block rows 1 (32) and 0 (16)
constexpr uint32_t kAA = 0;
constexpr uint32_t kAB = kAA + 2 * kRowsAA * 128;        // 28 KB
constexpr uint32_t kBL = kAB + 2 * kRowsAB * 128;        // + 12 KB: i side [L; Lq], 128 rows
constexpr uint32_t kRegionR = kBL + 2 * 128 * 128;       // + 32 KB = 72 KB
// after the A_kk MMAs: fp32 scratch and the bf16 T operand alias region R
constexpr uint32_t kSA = 0;
constexpr uint32_t kSAq = kSA + C * LT * 4;
constexpr uint32_t kST = kSAq + C * LT * 4;
constexpr uint32_t kSGb = kST + C * LT * 4;              // exact fallback: G of one block [16][128]
constexpr uint32_t kBT = 61440;                          // T bf16: 64 rows (t) x K = 64 (j)
// after the W / U MMAs: staging of W and U in the workspace layout (region R)
constexpr uint32_t kStgW = 0;
constexpr uint32_t kStgU = kStgW + C * LR * 2;
// region W: W / U MMA A operands, 128 rows (dk / dv) x K = 64 (t)
constexpr uint32_t kAW = kRegionR;
constexpr uint32_t kAU = kAW + 128 * 64 * 2;
constexpr uint32_t kTot = kAW;                           // block totals of g [4][128] (before region W is written)
constexpr uint32_t kGref = kAU + 128 * 64 * 2;           // G at rows 0, 16, 32, 48, 63: [5][128]
constexpr uint32_t kBeta = kGref + 5 * DK * 4;
constexpr uint32_t kGap = kBeta + C * 4;                 // per block max exponent gap (fp32 bits)
constexpr uint32_t kBar = kGap + 16;
constexpr uint32_t kHold = kBar + 24;  // bar[3]
constexpr uint32_t kBytes = kHold + 16;
constexpr size_t kSmem = kBytes + 1024;                  // + alignment of the swizzled tiles
constexpr uint32_t kTmemCols = 256;
constexpr float kGapMax = 80.f;
static_assert(kSGb + 16 * DK * 4 <= kBT && kBT + 64 * 128 <= kRegionR, "scratch must fit in region R");
static_assert(kStgU + 2 * kBUTile <= kRegionR && kStgW % 16 == 0 && kStgU % 16 == 0, "W / U staging");
static_assert(kSmem <= 113 * 1024, "two CTAs per SM");

// bulk copy shared -> global (bulk-group completion)
__device__ __forceinline__ void bulk_s2g(void* gdst, const void* ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(ssrc)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ uint32_t sw_off(int row, int k, int rows) {
  return (uint32_t)((k >> 6) * rows * 128 + row * 128 + ((((k & 63) >> 3) ^ (row & 7)) << 4) + (k & 7) * 2);
}
__device__ __forceinline__ uint32_t bf2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ void st_u32(uint8_t* base, uint32_t off, uint32_t v) {
  *reinterpret_cast<uint32_t*>(base + off) = v;
}
__device__ __forceinline__ float fexp(float x) { return __expf(x); }
__device__ __forceinline__ float2 exp2f2(float2 a, float2 b) {  // e^{a - b} per component
  return make_float2(fexp(a.x - b.x), fexp(a.y - b.y));
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return make_float2(a.x * b.x, a.y * b.y); }

__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

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

// a pair of elements kept packed in registers until used (16-bit: one word)
template <typename T>
struct Pair {
  using R = typename std::conditional<sizeof(T) == 4, float2, uint32_t>::type;
  static __device__ __forceinline__ R load(const T* p) { return *reinterpret_cast<const R*>(p); }
  static __device__ __forceinline__ float2 f2(R r) {
    if constexpr (sizeof(T) == 4) {
      return r;
    } else {
      const T* h = reinterpret_cast<const T*>(&r);
      return make_float2(to_f32<T>(h[0]), to_f32<T>(h[1]));
    }
  }
};
}  // namespace prep

// Phase timestamps of the first CTAs, compiled only into profiling builds
// (-DB2_KDA_PROFILE); the product build has no hook.
#ifdef B2_KDA_PROFILE
__device__ unsigned long long g_kda_prof[64][16];
__device__ unsigned long long g_kda_rprof[2][8][256];
#define B2_RPROF(k, c)                                                                       \
  do {                                                                                       \
    if (lane == 0 && warp == 0 && blockIdx.x < 2 && blockIdx.y == 0 && blockIdx.z == 0 && (c) < 256) \
      g_kda_rprof[rank][k][c] = globaltimer_ns();                                             \
  } while (0)
#define B2_PROF(i)                                                                  \
  do {                                                                              \
    if (threadIdx.x == 0 && blockIdx.x < 64 && blockIdx.y == 0 && blockIdx.z == 0)  \
      g_kda_prof[blockIdx.x][i] = globaltimer_ns();                                 \
  } while (0)
#else
#define B2_RPROF(k, c) \
  do {                 \
  } while (0)
#define B2_PROF(i) \
  do {             \
  } while (0)
#endif

template <typename T>
__global__ void __launch_bounds__(prep::kThreads, 2)
kda_prep_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                const float* __restrict__ g, const T* __restrict__ beta, float* __restrict__ ws, int B, int Tlen,
                int H, float scale, unsigned* __restrict__ err, const __grid_constant__ CUtensorMap tmV) {
  using namespace prep;
  // bf16 inputs: the chunk's v tile [64 t][128 d] arrives by TMA straight into
  // the U MMA's A operand (MN-major), and beta moves into T's columns
  // (U = T diag(beta) V, W = T diag(beta) K e^G), so no thread touches v.
  constexpr bool kTmaV = std::is_same<T, __nv_bfloat16>::value;
  using P2 = Pair<T>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  float* sTot = reinterpret_cast<float*>(sm + kTot);
  float* sGref = reinterpret_cast<float*>(sm + kGref);
  float* sBeta = reinterpret_cast<float*>(sm + kBeta);
  unsigned* sGap = reinterpret_cast<unsigned*>(sm + kGap);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kBar);
  uint32_t* hold = reinterpret_cast<uint32_t*>(sm + kHold);
  const int nc = Tlen / C;
  const int chunk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int dp = tid & 63, d0 = 2 * dp, I = tid >> 6, r0 = 16 * I;
  const int64_t row0 = ((int64_t)b * Tlen + (int64_t)chunk * C) * H + h;  // (b, t = chunk start, h)
  float* blk = ws + (((size_t)b * H + h) * nc + chunk) * kWsBlock;

  B2_PROF(0);
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    mbar_init(&bar[2], 1);
    fence_mbar_init();
    if constexpr (kTmaV) {
      // 3-D map {d, h, (b, t)}: two boxes of [64 t][1][64 d] (128-byte swizzle)
      mbar_arrive_expect_tx(&bar[2], 2u * C * 64 * 2);
      const int tv = b * Tlen + chunk * C;
#pragma unroll
      for (int hb = 0; hb < 2; ++hb)
        asm volatile(
            "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
                smem_u32(sm + kAU + hb * (C * 128))),
            "l"(&tmV), "r"(64 * hb), "r"(h), "r"(tv), "r"(smem_u32(&bar[2]))
            : "memory");
    }
  }
  if (tid < 4) sGap[tid] = 0u;
  if (warp == 0) {
    tc::tmem_alloc(hold, kTmemCols);
    tc::tmem_relinquish();
  }
  if (tid < C) sBeta[tid] = to_f32<T>(beta[row0 + (int64_t)tid * H]);

  // ---- 1. loads (all issued before any use), G ----
  typename P2::R kraw[16], qraw[16];
  float2 G[16];
#pragma unroll
  for (int r = 0; r < 16; ++r) {
    const int64_t gi = (row0 + (int64_t)(r0 + r) * H) * DK + d0;
    G[r] = *reinterpret_cast<const float2*>(g + gi);
    kraw[r] = P2::load(k + gi);
    qraw[r] = P2::load(q + gi);
  }
#pragma unroll
  for (int r = 1; r < 16; ++r) {
    G[r].x += G[r - 1].x;
    G[r].y += G[r - 1].y;
  }
  *reinterpret_cast<float2*>(sTot + I * DK + d0) = G[15];
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *hold;
  {
    float2 off = make_float2(0.f, 0.f);
    for (int J = 0; J < I; ++J) {
      const float2 tj = *reinterpret_cast<const float2*>(sTot + J * DK + d0);
      off.x += tj.x;
      off.y += tj.y;
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      G[r].x += off.x;
      G[r].y += off.y;
    }
    *reinterpret_cast<float2*>(sGref + I * DK + d0) = G[0];
    if (I == 3) *reinterpret_cast<float2*>(sGref + 4 * DK + d0) = G[15];
  }
  __syncthreads();  // sTot consumed (region W may be written from here on); sGref complete
  B2_PROF(1);

  // ---- 2. per-column constants of this block ----
  const float2 Gr0 = G[0];
  const float2 Gnx = *reinterpret_cast<const float2*>(sGref + (I + 1) * DK + d0);  // row 16 (I + 1), or 63
  const float2 Gl = *reinterpret_cast<const float2*>(sGref + 4 * DK + d0);
  {
    float gap = fmaxf(Gr0.x - Gnx.x, Gr0.y - Gnx.y);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) gap = fmaxf(gap, __shfl_xor_sync(0xffffffffu, gap, o));
    if (lane == 0) atomicMax(&sGap[I], __float_as_uint(fmaxf(gap, 0.f)));
  }
  const float2 zero2 = make_float2(0.f, 0.f);
  const float2 eG0 = exp2f2(Gr0, zero2);  // e^{G_r0}
  const float2 cD = exp2f2(Gr0, Gnx);     // e^{G_r0 - G_nx}, the diagonal j-side factor (>= 1)
  const float2 cKr = exp2f2(Gl, Gnx);     // e^{G_last - G_nx}
  float2 cOff[3];                          // e^{G_r0(I') - G_nx}, I' = I + 1 .. 3 (<= 1)
#pragma unroll
  for (int u = 0; u < 3; ++u)
    cOff[u] = I + 1 + u < 4 ? exp2f2(*reinterpret_cast<const float2*>(sGref + (I + 1 + u) * DK + d0), Gnx) : zero2;

  // ---- 3. operands of the A_kk / A_qk MMAs, the W operand, and scale Q e^G,
  // K e^{G_last - G} straight to the workspace ----
  __half* wsQg = ws_h(blk, kBQg);
  __half* wsKr = ws_h(blk, kBKr);
  float2 wk[16];  // beta K e^G (W operand); then beta V (U operand)
  // Swizzled operand addresses, hoisted: row t = r0 + r of a K-major tile
  // with `rows` rows sits at (d0 / 64) rows 128 + t 128, and this thread's
  // 16-byte chunk moves with t % 8 = r % 8 (r0 is a multiple of 16).
  uint32_t swz[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) swz[j] = ((((uint32_t)(d0 & 63) >> 3) ^ (uint32_t)j) << 4) + (uint32_t)(d0 & 7) * 2;
  // j-side rows of block row J: [A_kk operand region, first row]
  auto jrow = [&](int J) -> uint8_t* {
    const uint32_t region = J >= 2 ? kAA + (uint32_t)(d0 >> 6) * kRowsAA * 128 : kAB + (uint32_t)(d0 >> 6) * kRowsAB * 128;
    const int row0 = J == 3 ? 0 : J == 2 ? 64 : J == 1 ? 0 : 32;
    return sm + region + (row0 + r0) * 128;
  };
  uint8_t* const pL = sm + kBL + (uint32_t)(d0 >> 6) * 128 * 128 + r0 * 128;  // rows t (L); + 64 rows: Lq
  uint8_t* const pD = jrow(I);
  uint8_t* pO[3];
#pragma unroll
  for (int u = 0; u < 3; ++u) pO[u] = jrow(I + 1 + u < 4 ? I + 1 + u : 0);
#pragma unroll
  for (int r = 0; r < 16; ++r) {
    const int t = r0 + r;
    const uint32_t rs = (uint32_t)r * 128 + swz[r & 7];
    const float2 kk = P2::f2(kraw[r]);
    const float2 q2 = P2::f2(qraw[r]);
    const float2 sq = make_float2(q2.x * scale, q2.y * scale);
    const float2 e0 = exp2f2(G[r], Gr0);  // <= 1
    const float2 ej = exp2f2(Gnx, G[r]);  // <= 1
    const float2 lo = mul2(kk, e0), lq = mul2(sq, e0), kj = mul2(kk, ej);
    // i side: rows t (L) and 64 + t (Lq)
    st_u32(pL, rs, bf2(lo.x, lo.y));
    st_u32(pL + 64 * 128, rs, bf2(lq.x, lq.y));
    // j side: block row I (diagonal) and every later block row
    const float2 kd = mul2(kj, cD);
    st_u32(pD, rs, bf2(kd.x, kd.y));
#pragma unroll
    for (int u = 0; u < 3; ++u) {
      if (I + 1 + u >= 4) break;
      const float2 ko = mul2(kj, cOff[u]);
      st_u32(pO[u], rs, bf2(ko.x, ko.y));
    }
    *reinterpret_cast<__half2*>(wsQg + t * LR + d0) = __floats2half2_rn(lq.x * eG0.x, lq.y * eG0.y);
    *reinterpret_cast<__half2*>(wsKr + t * LR + d0) = __floats2half2_rn(kj.x * cKr.x, kj.y * cKr.y);
    const float bt = sBeta[t];
    wk[r] = kTmaV ? make_float2(lo.x * eG0.x, lo.y * eG0.y) : make_float2(bt * lo.x * eG0.x, bt * lo.y * eG0.y);
  }
  tc::fence_proxy_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  B2_PROF(2);

  // ---- 4. A_kk / A_qk MMAs (one thread) ----
  if (tid == 0) {
    tc::fence_after_sync();
    constexpr uint32_t idesc = tc::idesc_f16(128, 128, true);
#pragma unroll
    for (int s = 0; s < DK / 16; ++s) {
      const uint32_t ko = 2u * (s & 3);
      tc::mma_f16_ss(tmem, tc::desc_kmajor_sw128(sm + kAA + (s >> 2) * kRowsAA * 128) + ko,
                     tc::desc_kmajor_sw128(sm + kBL + (s >> 2) * 128 * 128) + ko, idesc, s != 0);
    }
#pragma unroll
    for (int s = 0; s < DK / 16; ++s) {
      const uint32_t ko = 2u * (s & 3);
      tc::mma_f16_ss(tmem + 128, tc::desc_kmajor_sw128(sm + kAB + (s >> 2) * kRowsAB * 128) + ko,
                     tc::desc_kmajor_sw128(sm + kBL + (s >> 2) * 128 * 128) + ko, idesc, s != 0);
    }
    tc::commit(&bar[0]);
  }
  // meanwhile: the W operand (rows d, K = t) of this thread's 16 t, then
  // beta V for the U operand (loads issued before the W stores)
  {
    typename P2::R vraw[16];
    if constexpr (!kTmaV) {
#pragma unroll
      for (int r = 0; r < 16; ++r) vraw[r] = P2::load(v + (row0 + (int64_t)(r0 + r) * H) * DV + d0);
    }
    uint32_t p0[8], p1[8];
#pragma unroll
    for (int r = 0; r < 16; r += 2) {
      p0[r / 2] = bf2(wk[r].x, wk[r + 1].x);
      p1[r / 2] = bf2(wk[r].y, wk[r + 1].y);
    }
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      *reinterpret_cast<uint4*>(sm + kAW + sw_off(d0, r0 + 8 * c, 128)) =
          make_uint4(p0[4 * c], p0[4 * c + 1], p0[4 * c + 2], p0[4 * c + 3]);
      *reinterpret_cast<uint4*>(sm + kAW + sw_off(d0 + 1, r0 + 8 * c, 128)) =
          make_uint4(p1[4 * c], p1[4 * c + 1], p1[4 * c + 2], p1[4 * c + 3]);
    }
    if constexpr (!kTmaV) {
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        const float bt = sBeta[r0 + r];
        const float2 vv = P2::f2(vraw[r]);
        wk[r] = make_float2(bt * vv.x, bt * vv.y);
      }
#pragma unroll
      for (int r = 0; r < 16; r += 2) {
        p0[r / 2] = bf2(wk[r].x, wk[r + 1].x);
        p1[r / 2] = bf2(wk[r].y, wk[r + 1].y);
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        *reinterpret_cast<uint4*>(sm + kAU + sw_off(d0, r0 + 8 * c, 128)) =
            make_uint4(p0[4 * c], p0[4 * c + 1], p0[4 * c + 2], p0[4 * c + 3]);
        *reinterpret_cast<uint4*>(sm + kAU + sw_off(d0 + 1, r0 + 8 * c, 128)) =
            make_uint4(p1[4 * c], p1[4 * c + 1], p1[4 * c + 2], p1[4 * c + 3]);
      }
    }
  }
  if (tid < DK / 2)
    *reinterpret_cast<float2*>(reinterpret_cast<uint8_t*>(blk) + kBGl + 4 * d0) = exp2f2(Gl, zero2);
  bool alive = mbar_wait(&bar[0], 0, err, 0xB2300001u);
  tc::fence_after_sync();
  // A_kk / A_qk scratch (aliases region R, which the MMAs just read)
  float* sA = reinterpret_cast<float*>(sm + kSA);
  float* sAq = reinterpret_cast<float*>(sm + kSAq);
  float* sT = reinterpret_cast<float*>(sm + kST);
  // (no clearing: the read-back below writes every lower entry, T reads only
  // lower entries of A_kk, and the A_qk store writes zeros above the diagonal)
  B2_PROF(3);

  // ---- 5. TMEM -> A_kk (times beta_i), A_qk: lane j = A-operand row; the
  // block row's 16 L columns (A_kk) and 16 Lq columns (A_qk) ----
  if (alive) {
    const int qd = warp & 3, half = warp >> 2;
    const int L = 32 * qd + lane;
    // (TMEM column base, block row, j of lane L) per warp; block rows with no lane here are skipped
    int Ib = -1, j = 0;
    uint32_t cb = 0;
    if (half == 0) {
      Ib = qd < 2 ? 3 : 2;
      j = qd < 2 ? L : L - 64;
      cb = 0;
    } else if (qd < 2) {
      Ib = qd == 0 ? 1 : 0;
      j = qd == 0 ? L : L - 32;
      cb = 128;
    }
    if (Ib >= 0) {
      const int ri = 16 * Ib;
      uint32_t va[16], vq[16];
      const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
      tmem_ld_x16(tmem + lane_off + cb + 16 * Ib, va);
      tmem_ld_x16(tmem + lane_off + cb + 64 + 16 * Ib, vq);
      tc::tmem_ld_wait();
      if (j < ri + 16) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if (j < ri + i) sA[(ri + i) * LT + j] = __uint_as_float(va[i]) * sBeta[ri + i];
          if (j <= ri + i) sAq[(ri + i) * LT + j] = __uint_as_float(vq[i]);
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  B2_PROF(4);
  // diagonal blocks whose exponent gap is beyond the bf16 / fp32 range of the
  // split factors: exact fp32 on CUDA cores (pairs j <= i of the block), with
  // the block's in-chunk G rebuilt from g (relative to its first row)
  for (int Ib = 0; Ib < 4; ++Ib) {
    if (__uint_as_float(sGap[Ib]) <= kGapMax) continue;
    float* sGb = reinterpret_cast<float*>(sm + kSGb);
    if (tid < DK) {
      float acc = 0.f;
      for (int r = 0; r < 16; ++r) {
        acc += g[(row0 + (int64_t)(16 * Ib + r) * H) * DK + tid];
        sGb[r * DK + tid] = acc;
      }
    }
    __syncthreads();
    for (int p = tid; p < 136; p += kThreads) {
      int i = 0, rem = p;
      while (rem > i) {
        rem -= i + 1;
        ++i;
      }
      const int ri = 16 * Ib + i, rj = 16 * Ib + rem;
      const T* ki = k + (row0 + (int64_t)ri * H) * DK;
      const T* qi = q + (row0 + (int64_t)ri * H) * DK;
      const T* kj = k + (row0 + (int64_t)rj * H) * DK;
      float akk = 0.f, aqk = 0.f;
      for (int d = 0; d < DK; ++d) {
        const float e = fexp(sGb[i * DK + d] - sGb[rem * DK + d]);
        const float kjd = to_f32<T>(kj[d]) * e;
        akk += to_f32<T>(ki[d]) * kjd;
        aqk += to_f32<T>(qi[d]) * kjd;
      }
      if (rj < ri) sA[ri * LT + rj] = akk * sBeta[ri];
      sAq[ri * LT + rj] = aqk * scale;
    }
    __syncthreads();
  }
  B2_PROF(5);

  // ---- 6 / 7. warps 0-1: T = (I + A_kk)^-1 on the diagonal 16 x 16 blocks,
  // column by column; warps 2-7 meanwhile: A_qk -> workspace (fp16, zeros
  // above the diagonal) and zeros of T above the diagonal blocks ----
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
  } else {
    __half* wsAq = ws_h(blk, kBAq);
    for (int e = tid - C; e < C * C / 2; e += kThreads - C) {
      const int r = (2 * e) / C, c2 = (2 * e) % C;
      const float a0 = c2 <= r ? sAq[r * LT + c2] : 0.f, a1 = c2 + 1 <= r ? sAq[r * LT + c2 + 1] : 0.f;
      *reinterpret_cast<__half2*>(wsAq + r * LA + c2) = __floats2half2_rn(a0, a1);
    }
    for (int e = tid - C; e < C * C; e += kThreads - C) {
      const int i = e / C, jc = e % C;
      if ((jc >> 4) > (i >> 4)) sT[i * LT + jc] = 0.f;
    }
  }
  __syncthreads();
  B2_PROF(6);
  // off-diagonal blocks of T on tf32 MMAs (m16n8k8, fp32 accumulate) in two
  // levels of the 2 x 2 block inverse
  //   T_BA = -T_BB A_BA T_AA    (A, B: the two halves of a diagonal block)
  // level 1 (16 x 16 halves, warps 0, 1):  blocks (1, 0) and (3, 2)
  // level 2 (32 x 32 halves, warps 0-3):   blocks (2, 0) (2, 1) (3, 0) (3, 1)
  // each as X_IJ = sum_M A_IM T_MJ (into sAq, no longer needed), then
  // T_IJ = -sum_M T_IM X_MJ.
  {
    const int gq = lane >> 2, tq = lane & 3;
    // X rows ri .. ri + 15, columns cj .. cj + 15, over m = mlo .. mhi - 1
    auto xpart = [&](int ri, int cj, int mlo, int mhi) {
      float x[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      for (int m0 = mlo; m0 < mhi; m0 += 8) {
        const uint32_t a0 = tf32(sA[(ri + gq) * LT + m0 + tq]), a1 = tf32(sA[(ri + gq + 8) * LT + m0 + tq]);
        const uint32_t a2 = tf32(sA[(ri + gq) * LT + m0 + tq + 4]), a3 = tf32(sA[(ri + gq + 8) * LT + m0 + tq + 4]);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
          mma_tf32(x[nt], a0, a1, a2, a3, tf32(sT[(m0 + tq) * LT + cj + 8 * nt + gq]),
                   tf32(sT[(m0 + tq + 4) * LT + cj + 8 * nt + gq]));
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        sAq[(ri + gq) * LT + cj + 8 * nt + 2 * tq] = x[nt][0];
        sAq[(ri + gq) * LT + cj + 8 * nt + 2 * tq + 1] = x[nt][1];
        sAq[(ri + gq + 8) * LT + cj + 8 * nt + 2 * tq] = x[nt][2];
        sAq[(ri + gq + 8) * LT + cj + 8 * nt + 2 * tq + 1] = x[nt][3];
      }
    };
    // T rows ri .. ri + 15, columns cj .. cj + 15 = -sum_{k = klo}^{ri + 15} T[ri][k] X[k][cj]
    auto ypart = [&](int ri, int cj, int klo) {
      float y[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      for (int kb = klo; kb < ri + 16; kb += 8) {
        const uint32_t a0 = tf32(sT[(ri + gq) * LT + kb + tq]), a1 = tf32(sT[(ri + gq + 8) * LT + kb + tq]);
        const uint32_t a2 = tf32(sT[(ri + gq) * LT + kb + tq + 4]), a3 = tf32(sT[(ri + gq + 8) * LT + kb + tq + 4]);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
          mma_tf32(y[nt], a0, a1, a2, a3, tf32(sAq[(kb + tq) * LT + cj + 8 * nt + gq]),
                   tf32(sAq[(kb + tq + 4) * LT + cj + 8 * nt + gq]));
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        sT[(ri + gq) * LT + cj + 8 * nt + 2 * tq] = -y[nt][0];
        sT[(ri + gq) * LT + cj + 8 * nt + 2 * tq + 1] = -y[nt][1];
        sT[(ri + gq + 8) * LT + cj + 8 * nt + 2 * tq] = -y[nt][2];
        sT[(ri + gq + 8) * LT + cj + 8 * nt + 2 * tq + 1] = -y[nt][3];
      }
    };
    if (warp < 2) {  // level 1: (1, 0) and (3, 2)
      const int ri = warp ? 48 : 16, cj = ri - 16;
      xpart(ri, cj, cj, ri);
      __syncwarp();
      ypart(ri, cj, ri);
    }
    __syncthreads();
    if (warp < 4) {  // level 2, X: rows 32 .. 63, columns 0 .. 31
      const int ri = 32 + 16 * (warp >> 1), cj = 16 * (warp & 1);
      xpart(ri, cj, cj, 32);
    }
    __syncthreads();
    if (warp < 4) {  // level 2, T: rows 32 .. 63, columns 0 .. 31
      const int ri = 32 + 16 * (warp >> 1), cj = 16 * (warp & 1);
      ypart(ri, cj, 32);
    }
    __syncthreads();
  }
  B2_PROF(7);
  // ---- 8. T (bf16) as the B operand: rows t, K = j ----
  {
    const int t = tid >> 2, c0 = 16 * (tid & 3);
    uint32_t pk[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float t0 = sT[t * LT + c0 + 2 * i], t1 = sT[t * LT + c0 + 2 * i + 1];
      if constexpr (kTmaV) {  // T diag(beta)
        t0 *= sBeta[c0 + 2 * i];
        t1 *= sBeta[c0 + 2 * i + 1];
      }
      pk[i] = bf2(t0, t1);
    }
    *reinterpret_cast<uint4*>(sm + kBT + sw_off(t, c0, 64)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    *reinterpret_cast<uint4*>(sm + kBT + sw_off(t, c0 + 8, 64)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
  }
  tc::fence_proxy_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  if (tid == 0 && alive) {
    tc::fence_after_sync();
    constexpr uint32_t idesc = tc::idesc_f16(128, 64, true);
#pragma unroll
    for (int s = 0; s < C / 16; ++s)
      tc::mma_f16_ss(tmem, tc::desc_kmajor_sw128(sm + kAW) + 2u * s, tc::desc_kmajor_sw128(sm + kBT) + 2u * s,
                     idesc, s != 0);
    if constexpr (kTmaV) {
      // v [t][d] as the MN-major A operand: 16 rows of t per k-step, the two
      // 64-column blocks of d 8 KB apart
      constexpr uint32_t idesc_v = tc::idesc_f16(128, 64, true, true, false);
      if (mbar_wait(&bar[2], 0, err, 0xB230000Cu)) {
#pragma unroll
        for (int s = 0; s < C / 16; ++s)
          tc::mma_f16_ss(tmem + 64, tc::smem_desc(sm + kAU + s * 16 * 128, C * 128, 1024, tc::kSwizzle128B),
                         tc::desc_kmajor_sw128(sm + kBT) + 2u * s, idesc_v, s != 0);
      }
    } else {
#pragma unroll
      for (int s = 0; s < C / 16; ++s)
        tc::mma_f16_ss(tmem + 64, tc::desc_kmajor_sw128(sm + kAU) + 2u * s, tc::desc_kmajor_sw128(sm + kBT) + 2u * s,
                       idesc, s != 0);
    }
    tc::commit(&bar[1]);
  }
  if (alive) alive = mbar_wait(&bar[1], 0, err, 0xB2300002u);
  tc::fence_after_sync();
  B2_PROF(8);
  // ---- 9. W^T, U^T (TMEM lane = dk / dv, column = t) -> W, U [t][d] fp16,
  // staged in shared memory in the workspace layout (region R is free once
  // the W / U MMAs are done) and written out by two bulk copies ----
  if (alive) {
    const int qd = warp & 3, half = warp >> 2;
    const int d = 32 * qd + lane;
    uint32_t va[32];
    // W [t][d] rows of LR; U [t][d % 64] in the tile of its 64 state columns
    __half* dst = half ? reinterpret_cast<__half*>(sm + kStgU + (d >> 6) * kBUTile) + (d & 63)
                       : reinterpret_cast<__half*>(sm + kStgW) + d;
    const int ld = half ? LUS : LR;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      tc::tmem_ld_32x32b_x32(tmem + ((uint32_t)(qd * 32) << 16) + 64u * half + 32u * c, va);
      tc::tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; ++i) dst[(32 * c + i) * ld] = __float2half_rn(__uint_as_float(va[i]));
    }
  }
  tc::fence_proxy_async_smem();
  tc::fence_before_sync();
  alive = __syncthreads_and(alive);
  if (tid == 0 && alive) {
    uint8_t* gb = reinterpret_cast<uint8_t*>(blk);
    bulk_s2g(gb + kBW, sm + kStgW, C * LR * 2);
    bulk_s2g(gb + kBU, sm + kStgU, 2 * kBUTile);
    asm volatile("cp.async.bulk.commit_group;\ncp.async.bulk.wait_group.read 0;" ::: "memory");
  }
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
  B2_PROF(9);
}

// ---------------------------------------------------------------------------
// Kernel B: state recurrence + outputs on a cluster of two CTAs per (b, h, 64
// state columns), 4 warps each; warp w of both CTAs owns the 16 state
// columns dv0 = v0 + 16 w .. dv0 + 15 for the whole sequence.  Columns of the
// state are independent (the transition acts on the Dk side only), so a warp
// never waits for another warp's state.  Everything runs on the transposed
// state S^T [Dv, Dk], held in fp32 m16n8 accumulator fragments, whose fp16
// copies are the A operands of the MMAs directly from registers.
//   state CTA (rank 0), the sequential chain:
//     V'^T = U^T - S^T W^T                 (16 x 64, K = 128)
//     S^T  = S^T o e^{G_last} + V'^T Kr    (16 x 128, K = 64)
//   output CTA (rank 1), off the chain:
//     O^T  = S^T Qg^T + V'^T A_qk^T        (16 x 64, K = 128 and K = 64, causal)
// Per chunk, each lane of a state warp sends its fp16 A fragments of S^T
// (before the update) and V'^T into the output CTA's shared memory
// (distributed shared memory, a two-slot ring per warp): the lanes stage them
// in a local slot, one lane bulk-copies the warp's 6 KB across, completing
// the slot's mbarrier transaction there; the output warp of the same columns
// reads them back lane for lane, re-arms the slot and releases it to the
// state warp.  (Per-lane remote stores cost 0.4 us per chunk on the state
// chain, 0.9 us with a release-arrive after them.)  Each CTA streams its part of the workspace block (W, Kr,
// e^{G_last} and its U tile; Qg and A_qk) through its own bulk-copy ring; the
// B operands come out of it by ldmatrix (Kr transposed).  S^T and V'^T enter
// the MMAs rounded to fp16 (10-bit mantissa); the state itself stays fp32.
// O leaves through a shared-memory tile so that each output row is one
// coalesced store.  Every wait is bounded; both CTAs meet at a cluster
// barrier before either exits, so no shared-memory access targets a CTA that
// has left.
// ---------------------------------------------------------------------------
constexpr int RW = 4;                 // warps per CTA
constexpr int RV = 16 * RW;           // state columns per CTA pair
constexpr int kRThreads = 32 * RW;
static_assert(RV == 64, "a cluster reads one 64-column U tile of the workspace");
constexpr int LO = RV + 8;            // output staging row stride (elements)
constexpr uint32_t kStage0 = kBStatePart + kBUTile;  // state CTA stage: W, Kr, e^{G_last}, U tile
constexpr uint32_t kStage1 = kBOutPart;              // output CTA stage: Qg, A_qk
constexpr int kNS0 = 4, kNS1 = 3;
constexpr int kSlotWords = 48;                         // per lane: S^T (8 x 4) + V'^T (4 x 4) fragments
constexpr uint32_t kSlotWarp = 32 * kSlotWords * 4;    // 6 KB
constexpr uint32_t kSlotBytes = RW * kSlotWarp;        // 24 KB per chunk
constexpr uint32_t kSlots1 = kNS1 * kStage1;           // output CTA: ring, then 2 slots, then staging
constexpr uint32_t kStaging1 = kSlots1 + 2 * kSlotBytes;
constexpr uint32_t kEnd1 = kStaging1 + C * LO * 4;     // (fp32 staging covers every output type)
constexpr uint32_t kSlots0 = kNS0 * kStage0;           // state CTA: ring, then 2 local staging slots
constexpr uint32_t kEnd0 = kSlots0 + 2 * kSlotBytes;
constexpr uint32_t kRBar = kEnd0 > kEnd1 ? kEnd0 : kEnd1;
// barriers: full0[kNS0], dempty[2][RW] (state CTA); full1[kNS1], dfull[2][RW] (output CTA)
constexpr uint32_t kRSmem = kRBar + 8 * (kNS0 + kNS1 + 4 * RW);
static_assert(kRSmem <= 227 * 1024, "kernel B shared memory");
static_assert(kStage0 % 16 == 0 && kStage1 % 16 == 0 && kSlots1 % 16 == 0, "bulk copy / vector alignment");

// bulk copy global -> shared (no multicast), completion on an mbarrier
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void r_load_stage0(uint8_t* st, const uint8_t* blk, int utile, uint64_t* bar) {
  mbar_arrive_expect_tx(bar, kStage0);
  bulk_g2s(st, blk, kBStatePart, bar);
  bulk_g2s(st + kBStatePart, blk + kBU + utile * kBUTile, kBUTile, bar);
}
__device__ __forceinline__ void r_load_stage1(uint8_t* st, const uint8_t* blk, uint64_t* bar) {
  mbar_arrive_expect_tx(bar, kStage1);
  bulk_g2s(st, blk + kBQg, kBOutPart, bar);
}

// ---- cluster helpers ----
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of this CTA's shared-memory location `p` in CTA `rank`
__device__ __forceinline__ uint32_t map_rank(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
// bulk copy of this CTA's shared memory into a partner CTA's (no multicast);
// the bytes count against the transaction count of the mbarrier `mbar` there
__device__ __forceinline__ void bulk_s2cluster(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst),
               "r"(smem_u32(src)), "r"(bytes), "r"(mbar)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// bounded wait that acquires at cluster scope (the arrivals come from the partner CTA)
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, unsigned* err, unsigned code) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((i & 255u) == 255u && globaltimer_ns() - t0 > kWaitNs) break;
  }
  atomicCAS(err, 0u, code);
  return false;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack_h2(uint32_t u) {
  return __half22float2(*reinterpret_cast<const __half2*>(&u));
}

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kRThreads, 1)
kda_recur_kernel(const float* __restrict__ ws, const float* __restrict__ s0, float* __restrict__ s_out,
                 T* __restrict__ o, int B, int Tlen, int H, unsigned* __restrict__ err) {
  extern __shared__ __align__(128) uint8_t smb[];
  uint64_t* full0 = reinterpret_cast<uint64_t*>(smb + kRBar);
  uint64_t* dempty = full0 + kNS0;   // [2][RW]
  uint64_t* full1 = dempty + 2 * RW;
  uint64_t* dfull = full1 + kNS1;    // [2][RW]
  const int nc = Tlen / C;
  const uint32_t rank = cluster_rank();
  const int utile = blockIdx.x >> 1, v0 = utile * RV, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3, mat = lane >> 3, r8 = lane & 7;
  const int dv0 = v0 + 16 * warp;
  const uint8_t* head = reinterpret_cast<const uint8_t*>(ws + ((size_t)b * H + h) * nc * kWsBlock);
  const size_t sbase = ((size_t)b * H + h) * DK * DV;

  if (tid == 0) {
    for (int i = 0; i < kNS0; ++i) mbar_init(&full0[i], 1);
    for (int i = 0; i < kNS1; ++i) mbar_init(&full1[i], 1);
    for (int i = 0; i < 2 * RW; ++i) {
      mbar_init(&dempty[i], 1);  // lane 0 of the output warp, after its warp read the slot
      mbar_init(&dfull[i], 1);   // the output warp's own expect_tx arrive + 6 KB of remote stores
    }
    fence_mbar_init();
  }
  cluster_sync();  // both CTAs' barriers initialised before any remote arrive

  bool alive = true;
  int c = 0;       // chunk the loop stopped at
  int issued = 0;  // chunks whose stage load thread 0 has issued
  if (rank == 0) {
    // ================================ state CTA ================================
    if (tid == 0)
      for (; issued < kNS0 && issued < nc; ++issued)
        r_load_stage0(smb + issued * kStage0, head + (size_t)issued * kWsBlockBytes, utile, &full0[issued]);
    // this lane's fragment slot in the output CTA: 12 16-byte groups, lane-interleaved
    const uint32_t slot_remote = map_rank(smb + kSlots1 + warp * kSlotWarp, 1);
    uint4* slot_stage = reinterpret_cast<uint4*>(smb + kSlots0 + warp * kSlotWarp) + lane;
    const uint32_t dfull_remote = map_rank(&dfull[warp], 1);
    // S^T fragments: n-tile nt covers dk 8 nt .. 8 nt + 7; e: (dv g | g + 8) x (dk 2 tq | 2 tq + 1)
    float S[16][4];
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int dk = 8 * nt + 2 * tq + (e & 1), dv = dv0 + g + 8 * (e >> 1);
        S[nt][e] = s0 ? s0[sbase + (size_t)dk * DV + dv] : 0.f;
      }
    for (; c < nc && alive; ++c) {
      const int sl = c % kNS0, ds = c & 1;
      const uint8_t* st = smb + sl * kStage0;
      // CTA-uniform verdict, so that no thread leaves the loop while others wait at a barrier
      B2_RPROF(0, c);
      alive = __syncthreads_and(mbar_wait(&full0[sl], (uint32_t)(c / kNS0) & 1u, err, 0xB2300003u));
      if (!alive) break;
      B2_RPROF(1, c);
      // this chunk's fragment slot in the output CTA (its previous hand-over,
      // two chunks back, is long consumed)
      const bool sent = mbar_wait_cluster(&dempty[ds * RW + warp], ((uint32_t)(c >> 1) & 1u) ^ 1u, err, 0xB230000Bu);
      uint4* stg = slot_stage + ds * (kSlotBytes / 16);
      const __half* sW = reinterpret_cast<const __half*>(st + kBW);
      const __half* sKr = reinterpret_cast<const __half*>(st + kBKr);
      const float* sGl = reinterpret_cast<const float*>(st + kBGl);
      const __half* sU = reinterpret_cast<const __half*>(st + kBStatePart);
      // S^T as fp16 A fragments, one per 16-wide dk step
      uint32_t sa[8][4];
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        sa[kk][0] = pack_h2(S[2 * kk][0], S[2 * kk][1]);
        sa[kk][1] = pack_h2(S[2 * kk][2], S[2 * kk][3]);
        sa[kk][2] = pack_h2(S[2 * kk + 1][0], S[2 * kk + 1][1]);
        sa[kk][3] = pack_h2(S[2 * kk + 1][2], S[2 * kk + 1][3]);
      }
      // acc = S^T W^T - U^T (= -V'^T), starting from -U^T read as C fragments
      float vp[8][4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        uint32_t u[4];
        ldsm_x4_trans(smem_u32(sU + (8 * (2 * p + (mat >> 1)) + r8) * LUS + 16 * warp + ((mat & 1) << 3)), u);
        const float2 a0 = unpack_h2(u[0]), a1 = unpack_h2(u[1]), a2 = unpack_h2(u[2]), a3 = unpack_h2(u[3]);
        vp[2 * p][0] = -a0.x;
        vp[2 * p][1] = -a0.y;
        vp[2 * p][2] = -a1.x;
        vp[2 * p][3] = -a1.y;
        vp[2 * p + 1][0] = -a2.x;
        vp[2 * p + 1][1] = -a2.y;
        vp[2 * p + 1][2] = -a3.x;
        vp[2 * p + 1][3] = -a3.y;
      }
      // V' MMAs; in their issue gaps: S^T o e^{G_last} (the MMAs read the
      // fp16 copy) and the staging of the S^T fragments for the output CTA
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          const int row = 16 * np + r8 + ((mat >> 1) << 3), col = 16 * kk + ((mat & 1) << 3);
          uint32_t bw[4];
          ldsm_x4(smem_u32(sW + row * LR + col), bw);
          const uint32_t w0[2] = {bw[0], bw[1]}, w1[2] = {bw[2], bw[3]};
          mma_16816<B2_F16>(vp[2 * np], sa[kk], w0);
          mma_16816<B2_F16>(vp[2 * np + 1], sa[kk], w1);
        }
#pragma unroll
        for (int nt = 2 * kk; nt < 2 * kk + 2; ++nt) {
          const float2 gl = *reinterpret_cast<const float2*>(sGl + 8 * nt + 2 * tq);
          S[nt][0] *= gl.x;
          S[nt][1] *= gl.y;
          S[nt][2] *= gl.x;
          S[nt][3] *= gl.y;
        }
        if (sent) stg[kk * 32] = make_uint4(sa[kk][0], sa[kk][1], sa[kk][2], sa[kk][3]);
      }
      // V'^T = -acc as fp16 A fragments over the chunk's 4 16-step blocks
      uint32_t va[4][4];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        va[kk][0] = pack_h2(-vp[2 * kk][0], -vp[2 * kk][1]);
        va[kk][1] = pack_h2(-vp[2 * kk][2], -vp[2 * kk][3]);
        va[kk][2] = pack_h2(-vp[2 * kk + 1][0], -vp[2 * kk + 1][1]);
        va[kk][3] = pack_h2(-vp[2 * kk + 1][2], -vp[2 * kk + 1][3]);
      }
      B2_RPROF(2, c);
      // S^T = S^T o e^{G_last} + V'^T Kr, staging V'^T in the MMA gaps
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int np = 0; np < 8; ++np) {
          uint32_t bk[4];
          ldsm_x4_trans(smem_u32(sKr + (16 * kk + r8 + ((mat & 1) << 3)) * LR + 16 * np + ((mat >> 1) << 3)), bk);
          const uint32_t k0[2] = {bk[0], bk[1]}, k1[2] = {bk[2], bk[3]};
          mma_16816<B2_F16>(S[2 * np], va[kk], k0);
          mma_16816<B2_F16>(S[2 * np + 1], va[kk], k1);
        }
        if (sent) stg[(8 + kk) * 32] = make_uint4(va[kk][0], va[kk][1], va[kk][2], va[kk][3]);
      }
      // hand the staged S^T / V'^T over: one bulk copy of the warp's 6 KB into
      // the output CTA, completing the slot's mbarrier transaction there
      if (sent) {
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0)
          bulk_s2cluster(slot_remote + ds * kSlotBytes, smb + kSlots0 + ds * kSlotBytes + warp * kSlotWarp, kSlotWarp,
                         dfull_remote + ds * RW * 8);
      }
      B2_RPROF(5, c);
      // every warp is done with stage sl (and agrees on the hand-over)
      alive = __syncthreads_and(sent);
      B2_RPROF(6, c);
      if (alive && tid == 0 && c + kNS0 < nc) {
        r_load_stage0(smb + sl * kStage0, head + (size_t)(c + kNS0) * kWsBlockBytes, utile, &full0[sl]);
        issued = c + kNS0 + 1;
      }
    }
    // the output warp has read the last two hand-overs, so no bulk copy out of
    // this CTA's staging slots is still in flight when the cluster exits
    for (int cc = c > 2 ? c - 2 : 0; cc < c && cc < nc; ++cc)
      mbar_wait_cluster(&dempty[(cc & 1) * RW + warp], (uint32_t)(cc >> 1) & 1u, err, 0xB230000Fu);
    if (s_out && alive) {
#pragma unroll
      for (int nt = 0; nt < 16; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int dk = 8 * nt + 2 * tq + (e & 1), dv = dv0 + g + 8 * (e >> 1);
          s_out[sbase + (size_t)dk * DV + dv] = S[nt][e];
        }
    }
  } else {
    // =============================== output CTA ================================
    T* sO = reinterpret_cast<T*>(smb + kStaging1);
    const uint32_t dempty_remote = map_rank(&dempty[warp], 0);
    const uint4* slot_local = reinterpret_cast<const uint4*>(smb + kSlots1 + warp * kSlotWarp) + lane;
    // arm both fragment slots for their first hand-over
    if (lane == 0)
      for (int i = 0; i < 2 && i < nc; ++i) mbar_arrive_expect_tx(&dfull[i * RW + warp], kSlotWarp);
    if (tid == 0)
      for (; issued < kNS1 && issued < nc; ++issued)
        r_load_stage1(smb + issued * kStage1, head + (size_t)issued * kWsBlockBytes, &full1[issued]);
    for (; c < nc && alive; ++c) {
      const int sl = c % kNS1, ds = c & 1;
      const uint8_t* st = smb + sl * kStage1;
      B2_RPROF(0, c);
      const bool got1 = mbar_wait(&full1[sl], (uint32_t)(c / kNS1) & 1u, err, 0xB230000Cu);
      B2_RPROF(1, c);
      const bool got = got1 && mbar_wait_cluster(&dfull[ds * RW + warp], (uint32_t)(c >> 1) & 1u, err, 0xB230000Du);
      B2_RPROF(2, c);
      alive = __syncthreads_and(got);
      B2_RPROF(3, c);
      if (!alive) break;
      const __half* sQg = reinterpret_cast<const __half*>(st + (kBQg - kBQg));
      const __half* sAq = reinterpret_cast<const __half*>(st + (kBAq - kBQg));
      uint32_t sa[8][4], va[4][4];
      const uint4* slot = slot_local + ds * (kSlotBytes / 16);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint4 x = slot[kk * 32];
        sa[kk][0] = x.x;
        sa[kk][1] = x.y;
        sa[kk][2] = x.z;
        sa[kk][3] = x.w;
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint4 x = slot[(8 + kk) * 32];
        va[kk][0] = x.x;
        va[kk][1] = x.y;
        va[kk][2] = x.z;
        va[kk][3] = x.w;
      }
      // the slot's contents are in registers: re-arm it for chunk c + 2 (the
      // state warp is told after the MMAs, when the release-arrive no longer
      // waits on outstanding memory operations)
      __syncwarp();
      if (lane == 0 && c + 2 < nc) mbar_arrive_expect_tx(&dfull[ds * RW + warp], kSlotWarp);
      float oa[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) oa[n][e] = 0.f;
      // O^T = S^T Qg^T
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          const int row = 16 * np + r8 + ((mat >> 1) << 3), col = 16 * kk + ((mat & 1) << 3);
          uint32_t bq[4];
          ldsm_x4(smem_u32(sQg + row * LR + col), bq);
          const uint32_t q0[2] = {bq[0], bq[1]}, q1[2] = {bq[2], bq[3]};
          mma_16816<B2_F16>(oa[2 * np], sa[kk], q0);
          mma_16816<B2_F16>(oa[2 * np + 1], sa[kk], q1);
        }
      }
      // O^T += V'^T A_qk^T: A_qk[i][j] = 0 for j > i, so key block kk only
      // reaches query blocks np >= kk
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          if (np < kk) continue;
          const int row = 16 * np + r8 + ((mat >> 1) << 3), col = 16 * kk + ((mat & 1) << 3);
          uint32_t ba[4];
          ldsm_x4(smem_u32(sAq + row * LA + col), ba);
          const uint32_t a0[2] = {ba[0], ba[1]}, a1[2] = {ba[2], ba[3]};
          mma_16816<B2_F16>(oa[2 * np], va[kk], a0);
          mma_16816<B2_F16>(oa[2 * np + 1], va[kk], a1);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(dempty_remote + ds * RW * 8);  // the slot is free again
      // O^T -> staging tile [t][dv], then coalesced rows of o
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = 8 * nt + 2 * tq + (e & 1), dvl = 16 * warp + g + 8 * (e >> 1);
          sO[t * LO + dvl] = from_f32<T>(oa[nt][e]);
        }
      __syncthreads();  // staging complete; every warp is done with stage sl
      if (tid == 0 && c + kNS1 < nc) {
        r_load_stage1(smb + sl * kStage1, head + (size_t)(c + kNS1) * kWsBlockBytes, &full1[sl]);
        issued = c + kNS1 + 1;
      }
      constexpr int PER = 16 / sizeof(T);  // elements per 16-byte store
      for (int e = tid; e < C * RV / PER; e += kRThreads) {
        const int t = e / (RV / PER), cc = e % (RV / PER);
        *reinterpret_cast<uint4*>(o + (((int64_t)b * Tlen + (int64_t)c * C + t) * H + h) * DV + v0 + PER * cc) =
            *reinterpret_cast<const uint4*>(sO + t * LO + PER * cc);
      }
      __syncthreads();  // staging tile read before the next chunk writes it
    }
  }
  // A CTA that gave up may leave bulk copies in flight into its own ring (the
  // stages of the chunks from c up to the last one issued): wait for them (bounded) before the
  // cluster exits.
  if (!alive && tid == 0) {
    const int ns = rank == 0 ? kNS0 : kNS1;
    uint64_t* fb = rank == 0 ? full0 : full1;
    for (int cc = c > 0 ? c - 1 : 0; cc < issued; ++cc)
      mbar_wait(&fb[cc % ns], (uint32_t)(cc / ns) & 1u, err, 0xB230000Eu);
  }
  cluster_sync();  // neither CTA leaves while the other may still address its shared memory
}
}  // namespace kda
}  // namespace b2

using namespace b2;

#ifdef B2_KDA_PROFILE
extern "C" __attribute__((visibility("default"))) int b2_kda_rprof_read(unsigned long long* host) {
  return (int)cudaMemcpyFromSymbol(host, kda::g_kda_rprof, sizeof(kda::g_kda_rprof));
}
extern "C" __attribute__((visibility("default"))) int b2_kda_prof_read(unsigned long long* host) {
  return (int)cudaMemcpyFromSymbol(host, kda::g_kda_prof, sizeof(kda::g_kda_prof));
}
#endif

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
  B2_CHECK_ARG(aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(g, 16) && aligned(o, 16) &&
                   aligned(workspace, 16),
               B2_ERR_ALIGN, "kda_fwd: q, k, v, g, o and the workspace must be 16-byte aligned");
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
  unsigned* err = device_error_word();
  B2_CHECK_ARG(err, B2_ERR_LAUNCH, "kda_fwd: no device error word");
  const dim3 ga((unsigned)(T / chunk), (unsigned)H, (unsigned)B);
  const dim3 gb(2 * (kda::DV / kda::RV), (unsigned)H, (unsigned)B);  // clusters of 2 along x
  CUtensorMap tmv;
  memset(&tmv, 0, sizeof(tmv));
  if (dtype == B2_BF16) {
    // v [B, T, H, Dv] as {d, h, (b, t)}
    const uint64_t dims[3] = {(uint64_t)Dv, (uint64_t)H, (uint64_t)(B * T)};
    const uint64_t strides[2] = {(uint64_t)Dv * 2, (uint64_t)H * Dv * 2};
    const uint32_t box[3] = {64, 1, (uint32_t)kda::C};
    B2_CHECK_ARG(make_tmap_3d(&tmv, v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_128B),
                 B2_ERR_INVALID, "kda_fwd: v tensor map: %s", b2_last_error());
  }
#define B2_KDA_LAUNCH(TY)                                                                                         \
  do {                                                                                                            \
    set_max_smem((const void*)kda::kda_prep_kernel<TY>, (int)kda::prep::kSmem);                                  \
    set_max_smem((const void*)kda::kda_recur_kernel<TY>, (int)kda::kRSmem);                                      \
    kda::kda_prep_kernel<TY><<<ga, kda::prep::kThreads, kda::prep::kSmem, st>>>(                                  \
        (const TY*)q, (const TY*)k, (const TY*)v, g, (const TY*)beta, ws, (int)B, (int)T, (int)H, scale, err, tmv); \
    kda::kda_recur_kernel<TY><<<gb, kda::kRThreads, kda::kRSmem, st>>>(                                         \
        ws, initial_state, final_state, (TY*)o, (int)B, (int)T, (int)H, err);                                    \
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

// W4A16 group-wise weight-only matmul: decode GEMV (M <= 16), the exact
// dequant export, the reference->GPTQ repack, and a generic per-output
// kernel for shapes outside the fast paths' constraints.
//
// Math (reference int4_matmul, triton_metal/codegen/_msl_templates.py:2716-2743):
//   out[m,n] = sum_k x[m,k] * (q[k,n] - z[g,n]) * s[g,n],  g = k / G.
//
// Decode GEMV design (HBM-bound, 0.5 byte of weight per MAC):
//   * Persistent: one CTA per SM owns a slab of <= 128 output columns and
//     streams it through a shared-memory ring with 2-D TMA copies (see
//     w4_gemv_stream_kernel below).
//   * In a stage, lane (g = lane/4, t = lane%4) reads packed words of GPTQ
//     row (4*quad + t), columns g and g + 8 of a 16-column MMA tile.
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
#include <string.h>

namespace b2 {

template <int DT>
struct Magic;
template <>
struct Magic<B2_F16> {
  static constexpr uint32_t base = 0x64006400u;   // (1024, 1024)
  static constexpr uint32_t base8 = 0x64086408u;  // (1032, 1032)
  static constexpr uint32_t one2 = 0x3C003C00u;   // (1.0, 1.0)
  static constexpr float bias = 1024.f;
};
template <>
struct Magic<B2_BF16> {
  static constexpr uint32_t base = 0x43004300u;   // (128, 128)
  static constexpr uint32_t base8 = 0x43084308u;  // (136, 136)
  static constexpr uint32_t one2 = 0x3F803F80u;   // (1.0, 1.0)
  static constexpr float bias = 128.f;
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

// Persistent streaming GEMV.  One CTA per SM owns a slab of columns
// [c0, c0 + w) (w <= 128, a multiple of 8).  The last warp (one elected
// lane) streams the slab through a ring of shared-memory stages with 2-D TMA
// tensor copies: one box of [G/8 rows x w columns] per quantisation group,
// plus one box holding the slab's whole [K/G x w] scale (and zero) block.
// Consumer warp w takes stage lane w % 8 (stages w%8, w%8 + 8, ...) and
// column half w / 8 (NCH = 2 halves for M <= 8, 1 for M <= 16): more warps
// per SM to issue the dequant + MMA work, which is what bounds this kernel
// once the copy engine keeps the weight stream in flight.
//
// Dequant is 7 integer ops per 32-bit word: each nibble pair becomes the
// exact fp16/bf16 value (bias + q) (bias = 1024 / 128) with one LOP3; the
// MMA then computes sum x*(bias+q) and the bias (and zero point) is removed
// per group with one extra MMA against a ones matrix, sum_k x:
//   sum_k x (q - z) = sum_k x (bias + q) - (bias + z) sum_k x.
// Both MMA products are exact and accumulate in fp32.
//
// Column mapping: in a 16-column MMA tile, A row g is smem column 2g and
// row g + 8 is column 2g + 1, so a lane fetches both words with one 64-bit
// shared load and both scales with one 32-bit load.
constexpr int kStageLanes = 8;
constexpr int kMaxColTiles = 16;  // 8-column tiles per CTA -> <= 128 columns
constexpr int kMaxMt = kMaxColTiles / 2;

struct GemvMaps {
  CUtensorMap w[2], s[2], z[2];  // [0]: CTAs with the wider slab, [1]: the rest
};

template <int DT>
__device__ __forceinline__ void biased_pairs(uint32_t w, uint32_t (&d)[4]) {
  d[0] = and_or(w, 0x000F000Fu, Magic<DT>::base);
  d[1] = and_or(w >> 4, 0x000F000Fu, Magic<DT>::base);
  d[2] = and_or(w >> 8, 0x000F000Fu, Magic<DT>::base);
  d[3] = and_or(w >> 12, 0x000F000Fu, Magic<DT>::base);
}

// fp16, symmetric: 5 ALU ops per word instead of 7.  Pairs 0 and 2 are
// (1024 + q) for nibbles (0, 4) and (2, 6); pairs 1 and 3 read nibbles (1, 5)
// and (3, 7) in place as (1024 + 16 q) and meet x / 16 (exact) in their k
// slots, so A * B = (64 + q) x there.  The bias MMA then uses the constant
// matrix c = 1032 (plain slots) | 1152 (x16 slots):
//   sum_k x (q - 8) = sum_k A B' - sum_k c_k B'.
__device__ __forceinline__ void pairs_f16_fast(uint32_t w, uint32_t (&d)[4]) {
  d[0] = and_or(w, 0x000F000Fu, 0x64006400u);
  d[1] = and_or(w, 0x00F000F0u, 0x64006400u);
  const uint32_t w8 = w >> 8;
  d[2] = and_or(w8, 0x000F000Fu, 0x64006400u);
  d[3] = and_or(w8, 0x00F000F0u, 0x64006400u);
}

// Shared bytes of the XS copy of x (M == 1): K / 8 rows of 16 B, 128-aligned.
__host__ __device__ inline int gemv_xs_bytes(int K) { return (K * 2 + 127) / 128 * 128; }

template <int NCH>
constexpr int gemv_threads() { return (kStageLanes * NCH + 1) * 32; }

// Two CTAs per SM when M <= 8, so that the CTAs of the next launch in a
// stream (programmatic dependent launch) can start streaming their weights
// while this launch's CTAs finish.
template <int NT>
constexpr int gemv_min_blocks() { return NT == 1 ? 2 : 1; }

// RQ = row quads per stage (G / 32); NT = 8-row tiles of M; NCH = column halves.
// XS (M == 1): each consumer warp copies the x rows of its own groups into
// shared memory once (cp.async, no CTA barrier) instead of re-reading them
// from L2 in every group round.
template <int DT, int NT, int RQ, int NCH, bool ZEROS, bool XS>
__global__ void __launch_bounds__(gemv_threads<NCH>(), gemv_min_blocks<NT>())
w4_gemv_stream_kernel(const __grid_constant__ GemvMaps maps, const uint16_t* __restrict__ x,
                      uint16_t* __restrict__ out, int M, int N, int K, int tiles_base, int tiles_rem,
                      int stages, int gps, unsigned* err) {
  using T = typename dtype_of<DT>::T;
  using T2 = typename dtype_of<DT>::T2;
  constexpr int R = 4 * RQ;                // weight rows (of 8 k) per stage
  constexpr int NCONS = kStageLanes * NCH;  // consumer warps
  constexpr int MPW = kMaxMt / NCH;         // m-tiles per consumer warp (max)
  extern __shared__ __align__(128) uint8_t smem[];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x;
  const int wide = b < tiles_rem ? 0 : 1;
  const int tile0 = b * tiles_base + min(b, tiles_rem);
  const int sw = (tiles_base + (wide == 0 ? 1 : 0)) * 8;  // slab width == smem row stride
  const int c0 = tile0 * 8;
  const int ncols = min(sw, N - c0);
  const int ngroups = K / (8 * R);
  const int max_sw = (tiles_base + (tiles_rem ? 1 : 0)) * 8;
  const int sblk = ((ngroups * max_sw * 2) + 127) / 128 * 128;  // scale block bytes
  const int slot_bytes = R * max_sw * 4;
  uint8_t* xsb = smem + sblk * (ZEROS ? 2 : 1);        // XS: x rows, 16 B each
  uint8_t* ring = xsb + (XS ? gemv_xs_bytes(K) : 0);
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + (size_t)stages * slot_bytes);
  uint64_t* empty = full + stages;
  uint64_t* sbar = empty + stages;
  // Let the next launch in the stream start as soon as SM resources allow;
  // it only streams weights until its own griddepcontrol.wait.
  asm volatile("griddepcontrol.launch_dependents;");
  if (ncols <= 0) return;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCH);
    }
    mbar_init(sbar, 1);
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == NCONS) {
    // ---------------- producer (one lane) ----------------
    if (lane != 0) return;
    const uint64_t pol = policy_evict_first();
    mbar_arrive_expect_tx(sbar, ngroups * sw * 2 * (ZEROS ? 2 : 1));
    tma_load_2d(smem, &maps.s[wide], c0, 0, sbar);
    if constexpr (ZEROS) tma_load_2d(smem + sblk, &maps.z[wide], c0, 0, sbar);
    // One TMA box covers gps consecutive groups (slots slot .. slot + gps - 1,
    // contiguous in shared memory) and completes on the first slot's barrier.
    for (int s = 0; s < ngroups; s += gps) {
      const int slot = s % stages;
      if (s >= stages)
        for (int j = 0; j < gps; ++j)
          if (!mbar_wait(&empty[slot + j], ((s / stages) - 1) & 1, err, 0xB2000001u)) return;
      mbar_arrive_expect_tx(&full[slot], gps * R * sw * 4);
      tma_load_2d_hint(ring + (size_t)slot * slot_bytes, &maps.w[wide], c0, s * R, &full[slot], pol);
    }
    return;
  }

  // ---------------- consumers ----------------
  const int g = lane >> 2, t = lane & 3;
  const int sid = warp % kStageLanes, ch = warp / kStageLanes;
  const int nmt = (ncols + 15) / 16;
  constexpr bool FAST = DT == B2_F16 && !ZEROS;
  // bias matrix of the correction MMA: all ones, or the (1032 | 1152)
  // pattern of the fp16 fast dequant (see pairs_f16_fast)
  const uint32_t ones[4] = {FAST ? 0x64086408u : Magic<DT>::one2, FAST ? 0x64086408u : Magic<DT>::one2,
                            FAST ? 0x64806480u : Magic<DT>::one2, FAST ? 0x64806480u : Magic<DT>::one2};
  float acc[MPW][NT][4];
#pragma unroll
  for (int a = 0; a < MPW; ++a)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][n][c] = 0.f;

  // x (and the output we overwrite) may be produced / still read by the
  // previous kernel in the stream: wait for it before touching either.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const uint4* xs4 = reinterpret_cast<const uint4*>(xsb);
  if constexpr (XS) {
    // the rows of this warp's groups sid, sid + 8, ... (row r of group s is x row s * R + r)
    const int nrow = ((ngroups - sid + kStageLanes - 1) / kStageLanes) * R;
    for (int i = lane; i < nrow; i += 32) {
      const int row = (sid + kStageLanes * (i / R)) * R + i % R;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(xsb + 16 * row)),
                   "l"(x + 8 * (size_t)row)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
    __syncwarp();
  }
  bool alive = mbar_wait(sbar, 0, err, 0xB2000003u);
  // ring slot and fill parity of group s, advanced without divisions (s
  // steps by the 8 stage lanes; stages is a multiple of 8 or covers every
  // group, and gps is a power of two)
  int slot = sid % stages;
  uint32_t fill_par = (uint32_t)(sid / stages) & 1u;
  for (int s = sid; s < ngroups && alive;
       s += kStageLanes, slot += kStageLanes, fill_par ^= (slot >= stages) ? 1u : 0u,
           slot -= (slot >= stages) ? stages : 0) {
    // x fragments of this group (L2 hits, or this warp's shared copy), loaded before the stage wait
    uint32_t bp[RQ][NT][4];
#pragma unroll
    for (int rq = 0; rq < RQ; ++rq) {
      const int row = s * R + 4 * rq + t;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const int m = g + 8 * n;
        uint4 xv = make_uint4(0, 0, 0, 0);
        if constexpr (XS) {
          if (m < M) xv = xs4[row];
        } else {
          if (m < M) xv = __ldg(reinterpret_cast<const uint4*>(x + (size_t)m * K + 8 * row));
        }
        x_pairs(xv, bp[rq][n]);
        if constexpr (FAST) {  // x / 16 in the slots where A holds 1024 + 16 q (exact)
          asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(bp[rq][n][1]) : "r"(0x2C002C00u));
          asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(bp[rq][n][3]) : "r"(0x2C002C00u));
        }
      }
    }
    // ds[n][.] = sum over the group's k of x[m], m = 8n + 2t (+1), via MMA
    float ds[NT][2][4];
#pragma unroll
    for (int rq = 0; rq < RQ; ++rq)
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const uint32_t b0[2] = {bp[rq][n][0], bp[rq][n][1]};
        const uint32_t b1[2] = {bp[rq][n][2], bp[rq][n][3]};
        if (rq == 0) {
          mma_16816_z<DT>(ds[n][0], ones, b0);
          mma_16816_z<DT>(ds[n][1], ones, b1);
        } else {
          mma_16816<DT>(ds[n][0], ones, b0);
          mma_16816<DT>(ds[n][1], ones, b1);
        }
      }
    const int slot0 = slot & ~(gps - 1);  // first slot of this group's box
    if (!mbar_wait(&full[slot0], fill_par, err, 0xB2000002u)) {
      alive = false;
      break;
    }
    // the box holds gps groups of R rows x sw columns back to back
    const uint32_t* wsm =
        reinterpret_cast<const uint32_t*>(ring + (size_t)slot0 * slot_bytes) + (size_t)(slot - slot0) * R * sw;
    const T* ssm = reinterpret_cast<const T*>(smem) + (size_t)s * sw;
    const T* zsm = reinterpret_cast<const T*>(smem + sblk) + (size_t)s * sw;
#pragma unroll
    for (int ip = 0; ip < MPW; ip += 2) {
      if (ch + NCH * ip < nmt) {
        // two m-tiles x two k-steps -> 4*NT independent MMA chains (the first
        // MMA of each chain starts from a zero accumulator)
        float cg[2][2][NT][4];
        uint2 wv[2][RQ];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int col = 16 * (ch + NCH * (ip + i)) + 2 * g;
#pragma unroll
          for (int rq = 0; rq < RQ; ++rq)
            wv[i][rq] = col < ncols ? *reinterpret_cast<const uint2*>(wsm + (4 * rq + t) * sw + col)
                                    : make_uint2(0, 0);
        }
#pragma unroll
        for (int rq = 0; rq < RQ; ++rq) {
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            uint32_t da[4], db[4];
            if constexpr (FAST) {
              pairs_f16_fast(wv[i][rq].x, da);
              pairs_f16_fast(wv[i][rq].y, db);
            } else {
              biased_pairs<DT>(wv[i][rq].x, da);
              biased_pairs<DT>(wv[i][rq].y, db);
            }
            const uint32_t a0[4] = {da[0], db[0], da[1], db[1]};
            const uint32_t a1[4] = {da[2], db[2], da[3], db[3]};
#pragma unroll
            for (int n = 0; n < NT; ++n) {
              const uint32_t b0[2] = {bp[rq][n][0], bp[rq][n][1]};
              const uint32_t b1[2] = {bp[rq][n][2], bp[rq][n][3]};
              if (rq == 0) {
                mma_16816_z<DT>(cg[i][0][n], a0, b0);
                mma_16816_z<DT>(cg[i][1][n], a1, b1);
              } else {
                mma_16816<DT>(cg[i][0][n], a0, b0);
                mma_16816<DT>(cg[i][1][n], a1, b1);
              }
            }
          }
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int col = 16 * (ch + NCH * (ip + i)) + 2 * g;
          const bool v = col < ncols;
          float2 sc = make_float2(0.f, 0.f);
          float2 bz = FAST ? make_float2(1.f, 1.f) : make_float2(Magic<DT>::bias + 8.f, Magic<DT>::bias + 8.f);
          if (v) {
            T2 sv = *reinterpret_cast<const T2*>(ssm + col);
            sc = make_float2(to_f32<T>(sv.x), to_f32<T>(sv.y));
            if constexpr (ZEROS) {
              T2 zv = *reinterpret_cast<const T2*>(zsm + col);
              bz = make_float2(Magic<DT>::bias + to_f32<T>(zv.x), Magic<DT>::bias + to_f32<T>(zv.y));
            }
          }
#pragma unroll
          for (int n = 0; n < NT; ++n) {
            const float d0 = ds[n][0][0] + ds[n][1][0], d1 = ds[n][0][1] + ds[n][1][1];
            float* ac = acc[ip + i][n];
            ac[0] += sc.x * ((cg[i][0][n][0] + cg[i][1][n][0]) - bz.x * d0);
            ac[1] += sc.x * ((cg[i][0][n][1] + cg[i][1][n][1]) - bz.x * d1);
            ac[2] += sc.y * ((cg[i][0][n][2] + cg[i][1][n][2]) - bz.y * d0);
            ac[3] += sc.y * ((cg[i][0][n][3] + cg[i][1][n][3]) - bz.y * d1);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }

  // Every stage (and the scale block) was waited for -> smem is free again,
  // unless a bounded wait ran out in some consumer warp: then copies may still
  // land in the ring, so no warp reuses it and no output is written (the
  // error word already records the timeout).  The barrier ORs the warps' flags.
  uint32_t any_dead;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.eq.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(any_dead)
      : "r"((uint32_t)alive), "n"(NCONS * 32)
      : "memory");
  if (any_dead) return;
  constexpr int CW = kMaxColTiles * 8;           // max slab width
  float* red = reinterpret_cast<float*>(smem);  // [stage lane][NT*8][CW]
  constexpr int RS = NT * 8 * CW;
#pragma unroll
  for (int i = 0; i < MPW; ++i) {
    const int col = 16 * (ch + NCH * i) + 2 * g;
    if (col < CW) {
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const int m = 8 * n + 2 * t;
        float* r = red + sid * RS;
        r[m * CW + col] = acc[i][n][0];
        r[(m + 1) * CW + col] = acc[i][n][1];
        r[m * CW + col + 1] = acc[i][n][2];
        r[(m + 1) * CW + col + 1] = acc[i][n][3];
      }
    }
  }
  asm volatile("bar.sync 1, %0;" ::"n"(NCONS * 32));
  for (int i = threadIdx.x; i < NT * 8 * CW; i += NCONS * 32) {
    const int m = i / CW, c = i % CW;
    if (m >= M || c >= ncols) continue;
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < kStageLanes; ++w) sum += red[w * RS + i];
    T r = from_f32<T>(sum);
    out[(size_t)m * N + c0 + c] = *reinterpret_cast<uint16_t*>(&r);
  }
}

constexpr int kSmemBudgetNT1 = 110 * 1024;  // two CTAs per SM (PDL overlap)
constexpr int kSmemBudgetNT2 = 227 * 1024;
constexpr int kMaxStages = 64;

struct GemvPlan {
  int grid, base, rem, stages, gps;
  size_t smem;
  bool xs;  // x staged per warp in shared memory (M == 1)
};

// Column-slab split over the SMs and shared-memory ring size for one shape.
static bool gemv_plan(int N, int K, int G, bool zeros, int nt, GemvPlan* p, int sms, bool xs = false) {
  const int budget = nt == 1 ? kSmemBudgetNT1 : kSmemBudgetNT2;
  // one CTA per SM; each owns a slab of <= 128 columns (8-column granules)
  const int tiles8 = N / 8;
  int ctas = sms;
  if (tiles8 < ctas) ctas = tiles8;
  int base = tiles8 / ctas, rem = tiles8 % ctas;
  if (base + (rem ? 1 : 0) > kMaxColTiles) {  // very wide N: more CTAs than SMs
    ctas = (tiles8 + kMaxColTiles - 1) / kMaxColTiles;
    base = tiles8 / ctas;
    rem = tiles8 % ctas;
  }
  const int max_sw = (base + (rem ? 1 : 0)) * 8;
  const int rows = G / 8, ngroups = K / G;
  if (ngroups > 256) return false;  // TMA box dimension limit of the scale block
  const size_t sblk = ((size_t)ngroups * max_sw * 2 + 127) / 128 * 128;
  const size_t slot = (size_t)rows * max_sw * 4;
  const size_t fixed = sblk * (zeros ? 2 : 1) + (xs ? gemv_xs_bytes(K) : 0);
  int stages = (int)((budget - fixed - 256) / (slot + 16));
  if (stages > kMaxStages) stages = kMaxStages;
  // Consumer warp w takes groups w, w + 8, ... and waits on ring slot
  // s % stages with parity (s / stages) & 1.  A parity wait one phase ahead
  // of the slot's current phase returns at once, so a slot must only ever be
  // reused by the warp that used it before (which has already waited for the
  // previous fill): stages is a multiple of the 8 stage lanes, unless every
  // group has its own slot.
  if (stages >= ngroups) stages = ngroups;
  else stages -= stages % kStageLanes;
  if (stages < 1) return false;
  // groups per TMA box: the largest of 4, 2, 1 that divides the ring and the
  // group count and keeps the box within 256 rows (fewer, larger boxes
  // stream faster: 5 KB boxes ran ~1.5x slower than 10 KB ones)
  p->gps = 1;
  for (int gps = 4; gps > 1; gps >>= 1)
    if (stages % gps == 0 && ngroups % gps == 0 && rows * gps <= 256) {
      p->gps = gps;
      break;
    }
  size_t total = fixed + (size_t)stages * (slot + 16) + 16;
  const size_t red = (size_t)kStageLanes * nt * 8 * kMaxColTiles * 8 * 4;
  if (total < red) total = red;
  p->grid = ctas;
  p->base = base;
  p->rem = rem;
  p->stages = stages;
  p->smem = total;
  return total <= (size_t)budget;
}

// Plan used for an M-row call: with M == 1 the x copy in shared memory is
// taken when it leaves the ring as deep as without it.
static bool gemv_choose(int M, int N, int K, int G, bool zeros, int sms, GemvPlan* p) {
  const int nt = M <= 8 ? 1 : 2;
  if (!gemv_plan(N, K, G, zeros, nt, p, sms)) return false;
  p->xs = false;
  GemvPlan q;
  if (M == 1 && gemv_plan(N, K, G, zeros, nt, &q, sms, true) && q.stages == p->stages) {
    *p = q;
    p->xs = true;
  }
  return true;
}

template <int DT, int NT, int RQ, int NCH, bool ZEROS>
static int launch_stream(const void* x, const void* w, void* out, const void* s, const void* z, int M, int N, int K,
                         int G, cudaStream_t st) {
  GemvPlan p;
  if (!gemv_choose(M, N, K, G, ZEROS, num_sms(), &p)) return B2_ERR_UNSUPPORTED;
  unsigned* err = device_error_word();
  if (!err) {
    set_error("w4_gemv: cannot resolve the device error word");
    return B2_ERR_LAUNCH;
  }
  const int ngroups = K / G, rows = G / 8;
  const CUtensorMapDataType sdt = DT == B2_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  GemvMaps maps;
  memset(&maps, 0, sizeof(maps));
  const int widths[2] = {(p.base + 1) * 8, p.base * 8};
  for (int i = 0; i < 2; ++i) {
    const int wdt = widths[i];
    if (wdt == 0 || (i == 0 && p.rem == 0)) continue;
    if (!make_tmap_2d(&maps.w[i], w, CU_TENSOR_MAP_DATA_TYPE_UINT32, N, K / 8, (uint64_t)N * 4, wdt, rows * p.gps) ||
        !make_tmap_2d(&maps.s[i], s, sdt, N, ngroups, (uint64_t)N * 2, wdt, ngroups) ||
        (ZEROS && !make_tmap_2d(&maps.z[i], z, sdt, N, ngroups, (uint64_t)N * 2, wdt, ngroups)))
      return B2_ERR_INVALID;
  }
  auto kern = w4_gemv_stream_kernel<DT, NT, RQ, NCH, ZEROS, false>;
  if constexpr (NT == 1)
    if (p.xs) kern = w4_gemv_stream_kernel<DT, NT, RQ, NCH, ZEROS, true>;
  set_max_smem((const void*)kern, (int)p.smem);
  // Programmatic dependent launch: may overlap the previous kernel of the
  // stream; the kernel itself orders every dependent access after
  // griddepcontrol.wait (a no-op when the previous kernel did not trigger).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(gemv_threads<NCH>());
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, maps, (const uint16_t*)x, (uint16_t*)out, M, N, K, p.base, p.rem, p.stages, p.gps,
                     err);
  return launch_status("w4_gemv");
}

template <int DT, int RQ>
static int gemv_nt(const void* x, const void* w, void* out, const void* s, const void* z, int M, int N, int K, int G,
                   cudaStream_t st) {
  if (M <= 8)
    return z ? launch_stream<DT, 1, RQ, 1, true>(x, w, out, s, z, M, N, K, G, st)
             : launch_stream<DT, 1, RQ, 1, false>(x, w, out, s, z, M, N, K, G, st);
  return z ? launch_stream<DT, 2, RQ, 1, true>(x, w, out, s, z, M, N, K, G, st)
           : launch_stream<DT, 2, RQ, 1, false>(x, w, out, s, z, M, N, K, G, st);
}

template <int DT>
static int gemv_dispatch(const void* x, const void* w, void* out, const void* s, const void* z, int M, int N, int K,
                         int G, cudaStream_t st) {
  switch (G / 32) {
    case 1: return gemv_nt<DT, 1>(x, w, out, s, z, M, N, K, G, st);
    case 2: return gemv_nt<DT, 2>(x, w, out, s, z, M, N, K, G, st);
    case 4: return gemv_nt<DT, 4>(x, w, out, s, z, M, N, K, G, st);
    case 8: return gemv_nt<DT, 8>(x, w, out, s, z, M, N, K, G, st);
    default: return B2_ERR_UNSUPPORTED;
  }
}

// Layout constraints of the streaming GEMV (TMA: 16-byte aligned rows/boxes).
static bool gemv_ok(const void* x, const void* w, const void* s, const void* z, int64_t M, int64_t N, int64_t K,
                    int64_t G) {
  const int64_t spg = G / 32;
  return M >= 1 && M <= 16 && N % 8 == 0 && K % G == 0 && G % 32 == 0 &&
         (spg == 1 || spg == 2 || spg == 4 || spg == 8) && K / G <= 256 && aligned(x, 16) && aligned(w, 16) &&
         aligned(s, 16) && (!z || aligned(z, 16));
}


}  // namespace b2

using namespace b2;

// Implemented in wxa16_gemm_sm100.cu: tcgen05 prefill GEMM for M > 16.
int b2_detail_w4_gemm(const void* x, const void* w, void* out, const void* s, const void* z,
                      int64_t M, int64_t N, int64_t K, int64_t G, int dtype, cudaStream_t st);

namespace b2 {
// quant_f32.cu: fp32 activations / scales / zeros / output on CUDA cores
int b2_detail_quant_f32(int layout, const void* x, const void* w, void* out, const void* s, const void* z,
                        int64_t M, int64_t N, int64_t K, int64_t G, cudaStream_t st);
}  // namespace b2

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
  B2_CHECK_ARG(dtype == B2_F16 || dtype == B2_BF16 || dtype == B2_F32, B2_ERR_DTYPE,
               "int4_matmul: dtype %d unsupported", dtype);
  B2_CHECK_ARG(M * N < (1ll << 31) && K * N / 8 < (1ll << 31), B2_ERR_UNSUPPORTED, "int4_matmul: too large");
  if (M == 0) return B2_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == B2_F32) return b2_detail_quant_f32(0, input, weight, output, scales, zeros, M, N, K, group_size, st);
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

// Host plan of the streaming decode GEMV for one shape, for tests and tools
// (no device work): info = {grid, slab tiles (8 columns) per CTA, CTAs with
// one extra tile, ring stages, groups per TMA box, shared-memory bytes}.
extern "C" int b2_w4_gemv_plan(int64_t M, int64_t N, int64_t K, int64_t group_size, int zeros, int sms,
                               int64_t* info) {
  B2_CHECK_ARG(info && sms > 0 && M > 0 && N > 0 && K > 0 && group_size > 0, B2_ERR_INVALID,
               "w4_gemv_plan: bad arguments");
  const int64_t spg = group_size / 32;
  if (!(M <= 16 && N % 8 == 0 && K % group_size == 0 && group_size % 32 == 0 &&
        (spg == 1 || spg == 2 || spg == 4 || spg == 8) && K / group_size <= 256 && N < (1ll << 31) &&
        K < (1ll << 31)))
    return B2_ERR_UNSUPPORTED;
  GemvPlan p;
  if (!gemv_choose((int)M, (int)N, (int)K, (int)group_size, zeros != 0, sms, &p)) return B2_ERR_UNSUPPORTED;
  info[0] = p.grid;
  info[1] = p.base;
  info[2] = p.rem;
  info[3] = p.stages;
  info[4] = p.gps;
  info[5] = (int64_t)p.smem;
  return B2_OK;
}

// Decode attention (one query token per head) over a contiguous or paged KV
// cache, split-KV ("flash decoding"), sm_100a.
//
// Reference kernels this replaces (triton_metal/codegen/_msl_templates.py):
//   kv_cache_attention (:1949-2063), gqa_attention (:2064-2164),
//   batched_kv_decode (:2167-2278), paged_attention (:2279-2404),
//   multi_head_paged_attention (:2405-2532), fp16_kv_attention (:2533-2627),
//   sliding_window_attention (:3335-3431), rope_attention (:1770-1887).
// Those compute one (batch, head) per threadgroup in three passes that
// recompute Q.K (max, sum, weighted V).  Here:
//   * one CTA per (KV split, kv head, batch) handles all Hq/Hkv query heads of
//     its kv head, so each K/V row is read from HBM exactly once;
//   * 64-key tiles are staged in shared memory (fp32) and the query heads are
//     spread over the 4 warps: lane = key for the scores (one pass, online
//     softmax with warp-shuffle max/sum), lane = head dimension for P.V;
//   * splits write (m, l, unnormalised O) partials that a second kernel
//     merges (O = sum_s e^{m_s - M} O_s / sum_s e^{m_s - M} l_s); with one split
//     the CTA writes O directly.
// Layouts: q [B, Hq, D]; contiguous K/V [B, Hkv, S, D] with element strides
// (b, h, s); paged K/V [n_pages, page_size, Hkv, D] with page_table
// [B, max_pages] (logical -> physical page); seq_lens [B].  The KV dtype may
// differ from the query dtype (fp16 KV with fp32 queries).
// Options: q_pos [B] (default seq_len - 1) and window W > 0 restrict the
// keys to [max(0, q_pos + 1 - W), min(q_pos + 1, seq_len)) (sliding window);
// rope freqs [D/2] rotate q at q_pos and key j at j, pairs (2d, 2d + 1) by
// angle pos * freqs[d], before the dot products (V is not rotated).
#include "b2_common.cuh"
#include <type_traits>

namespace b2 {
namespace dec {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int TK = 64;          // keys per tile
constexpr int kMaxD = 256;
constexpr int kMaxRep = 16;     // query heads per kv head

struct Params {
  const void *q, *k, *v;
  void* o;
  const int32_t* page_table;
  const int32_t* seq_lens;
  float* ws;  // partials: [B, Hq, nsplit] x (m, l, D values)
  int B, Hq, Hkv, D, page_size, max_pages, nsplit, split_len;
  int64_t ks[3], vs[3];  // contiguous: (b, h, s) element strides; paged: (page, token, head)
  float scale;
  const int32_t* q_pos;  // [B] or null (seq_len - 1)
  int window;            // > 0: sliding window
  int cap;               // keys a sequence may reach: max_seq_len (<= max_pages * page_size when paged)
  const float* rope;     // [D/2] RoPE frequencies or null
};

// Key range [lo, hi) of sequence b and its query position.
__device__ __forceinline__ void key_range(const Params& p, int b, int& lo, int& hi, int& qp) {
  // seq_lens[b] beyond the caller's max_seq_len is clamped to it: the splits
  // only cover max_seq_len keys and a paged row only max_pages pages.
  const int len = min(p.seq_lens[b], p.cap);
  qp = p.q_pos ? p.q_pos[b] : len - 1;
  lo = 0;
  hi = len;
  if (p.window > 0) {
    lo = max(0, qp + 1 - p.window);
    hi = min(qp + 1, len);
  }
}

// cos / sin of pos * f: the angle is formed and reduced in double precision
// (positions reach 10^5 radians), the result rounded to float.
__device__ __forceinline__ float2 rope_cs(double pos, float f) {
  double sn, cs;
  sincos(pos * (double)f, &sn, &cs);
  return make_float2((float)cs, (float)sn);
}

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

template <typename TQ, typename TKV, bool PAGED>
__global__ void __launch_bounds__(kThreads)
decode_split_kernel(const Params p) {
  extern __shared__ float sm[];
  const int D = p.D, LDK = D + 1;
  float* sQ = sm;                    // [rep][D]
  float* sK = sQ + kMaxRep * D;      // [TK][D + 1]
  float* sV = sK + TK * LDK;         // [TK][D + 1]
  float* sP = sV + TK * LDK;         // [kWarps][TK]
  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rep = p.Hq / p.Hkv;
  int lo, hi, qp;
  key_range(p, b, lo, hi, qp);
  const int s0 = lo + split * p.split_len, s1 = min(hi, s0 + p.split_len);

  for (int e = tid; e < rep * D; e += kThreads) {
    const int hh = e / D, d = e % D;
    const TQ* qrow = (const TQ*)p.q + ((int64_t)b * p.Hq + hk * rep + hh) * D;
    float val = ldf(qrow + d);
    if (p.rope) {
      const int pr = d >> 1;
      const float2 cs = rope_cs((double)qp, p.rope[pr]);
      const float a = ldf(qrow + 2 * pr), c = ldf(qrow + 2 * pr + 1);
      val = (d & 1) ? a * cs.y + c * cs.x : a * cs.x - c * cs.y;
    }
    sQ[e] = val * p.scale;
  }
  // per-warp state for its query heads hh = warp, warp + 4, ...
  constexpr int kHPW = kMaxRep / kWarps;       // <= 4 heads per warp
  constexpr int kDPL = kMaxD / 32;             // <= 8 head-dim values per lane
  float m[kHPW], l[kHPW], acc[kHPW][kDPL];
#pragma unroll
  for (int i = 0; i < kHPW; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int j = 0; j < kDPL; ++j) acc[i][j] = 0.f;
  }
  const TKV* kb = (const TKV*)p.k;
  const TKV* vb = (const TKV*)p.v;
  for (int t0 = s0; t0 < s1; t0 += TK) {
    __syncthreads();  // previous tile consumed
    for (int e = tid; e < TK * D; e += kThreads) {
      const int j = e / D, d = e % D, pos = t0 + j;
      float kv = 0.f, vv = 0.f;
      if (pos < s1) {
        int64_t ko, vo;
        if constexpr (PAGED) {
          const int pg = p.page_table[(int64_t)b * p.max_pages + pos / p.page_size];
          const int off = pos % p.page_size;
          ko = pg * p.ks[0] + off * p.ks[1] + hk * p.ks[2] + d;
          vo = pg * p.vs[0] + off * p.vs[1] + hk * p.vs[2] + d;
        } else {
          ko = b * p.ks[0] + hk * p.ks[1] + (int64_t)pos * p.ks[2] + d;
          vo = b * p.vs[0] + hk * p.vs[1] + (int64_t)pos * p.vs[2] + d;
        }
        kv = ldf(kb + ko);
        vv = ldf(vb + vo);
      }
      sK[j * LDK + d] = kv;
      sV[j * LDK + d] = vv;
    }
    __syncthreads();
    if (p.rope) {  // rotate the staged keys in place at their positions
      for (int e = tid; e < TK * (D / 2); e += kThreads) {
        const int j = e / (D / 2), pr = e % (D / 2);
        const float2 cs = rope_cs((double)(t0 + j), p.rope[pr]);
        float* kp = sK + j * LDK + 2 * pr;
        const float a = kp[0], c = kp[1];
        kp[0] = a * cs.x - c * cs.y;
        kp[1] = a * cs.y + c * cs.x;
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < kHPW; ++i) {
      const int hh = warp + kWarps * i;
      if (hh >= rep) break;
      // scores of keys lane and lane + 32
      float sc[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int j = lane + 32 * u;
        float dot = 0.f;
        for (int d = 0; d < D; ++d) dot += sQ[hh * D + d] * sK[j * LDK + d];
        sc[u] = (t0 + j < s1) ? dot : -INFINITY;
      }
      float tmax = fmaxf(sc[0], sc[1]);
#pragma unroll
      for (int off = 16; off; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
      const float mn = fmaxf(m[i], tmax);
      const float alpha = __expf(m[i] - mn);  // m = -inf -> 0
      const float p0 = __expf(sc[0] - mn), p1 = __expf(sc[1] - mn);
      float ts = p0 + p1;
#pragma unroll
      for (int off = 16; off; off >>= 1) ts += __shfl_xor_sync(0xffffffffu, ts, off);
      l[i] = l[i] * alpha + ts;
      m[i] = mn;
      float* pw = sP + warp * TK;
      pw[lane] = p0;
      pw[lane + 32] = p1;
      __syncwarp();
#pragma unroll
      for (int jd = 0; jd < kDPL; ++jd) acc[i][jd] *= alpha;
      for (int j = 0; j < TK; ++j) {
        const float pj = pw[j];
#pragma unroll
        for (int jd = 0; jd < kDPL; ++jd) {
          const int d = lane + 32 * jd;
          if (d < D) acc[i][jd] += pj * sV[j * LDK + d];
        }
      }
      __syncwarp();
    }
  }
  // write the result (one split) or the partial (m, l, O)
#pragma unroll
  for (int i = 0; i < kHPW; ++i) {
    const int hh = warp + kWarps * i;
    if (hh >= rep) break;
    const int hq = hk * rep + hh;
    if (p.nsplit == 1) {
      const float inv = l[i] > 0.f ? 1.f / l[i] : 0.f;
#pragma unroll
      for (int jd = 0; jd < kDPL; ++jd) {
        const int d = lane + 32 * jd;
        if (d < D) stf((TQ*)p.o + ((int64_t)b * p.Hq + hq) * D + d, acc[i][jd] * inv);
      }
    } else {
      float* w = p.ws + (((int64_t)b * p.Hq + hq) * p.nsplit + split) * (D + 2);
      if (lane == 0) {
        w[0] = m[i];
        w[1] = l[i];
      }
#pragma unroll
      for (int jd = 0; jd < kDPL; ++jd) {
        const int d = lane + 32 * jd;
        if (d < D) w[2 + d] = acc[i][jd];
      }
    }
  }
}

template <typename TQ>
__global__ void decode_combine_kernel(const Params p) {
  const int bh = blockIdx.x;  // b * Hq + hq
  const int D = p.D;
  const float* w = p.ws + (int64_t)bh * p.nsplit * (D + 2);
  float M = -INFINITY;
  for (int s = 0; s < p.nsplit; ++s) M = fmaxf(M, w[s * (D + 2)]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float num = 0.f, den = 0.f;
    for (int s = 0; s < p.nsplit; ++s) {
      const float* ws = w + s * (D + 2);
      if (ws[0] == -INFINITY) continue;  // empty split
      const float f = __expf(ws[0] - M);
      num += f * ws[2 + d];
      den += f * ws[1];
    }
    stf((TQ*)p.o + (int64_t)bh * D + d, den > 0.f ? num / den : 0.f);
  }
}


// ---------------------------------------------------------------------------
// Tensor-core path: 16-bit q and KV cache of the same type, D in {64, 128, 256}.
//
// A CTA streams its split of one (batch, kv head) through a STAGES-deep ring
// of 64-key K/V tiles filled by 16-byte cp.async (zero-filled past the
// sequence end, so every tile is the same shape).  Tiles are stored
// row-major with the 16-byte chunks of a row XOR-swizzled by (row & 7) so the
// 8 row addresses of an ldmatrix hit 8 different bank groups.  Warp w owns
// keys [16w, 16w + 16) of every tile and keeps its own online-softmax state:
//   S[16 x 16]  = Q[16 x D] . K_w^T       (rows = the rep query heads, zero
//                                          padded to 16; mma m16n8k16)
//   O[16 x D]  += exp2(S - m) . V_w        (P re-used from the accumulator
//                                          registers as the A operand)
// The 4 warps' (m, l, O) are merged through shared memory at the end.
// Per 64-key tile each warp issues 16 ldmatrix + 32 MMAs for D = 128, far
// below the ~1400 SM cycles the tile's 32 KB take at the CTA's share of HBM
// bandwidth, so the kernel is bound by the copy stream.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit_grp() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_grp() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (std::is_same<T, __half>::value) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

template <int D>
struct TcCfg {
  static constexpr int kStages = D == 64 ? 6 : (D == 128 ? 3 : 3);
  static constexpr int kRowBytes = D * 2;
  static constexpr int kTileBytes = TK * kRowBytes;           // one of K or V
  static constexpr int kQBytes = 16 * kRowBytes;
  static constexpr int kSmem = kQBytes + kStages * 2 * kTileBytes;
  static constexpr int kChunks = D / 8;                       // 16-byte chunks per row
  static constexpr int kRowsPerPass = kThreads / kChunks;
  static_assert(kWarps * D * 16 * 4 + 2 * kWarps * 16 * 4 <= kStages * 2 * kTileBytes, "merge buffer");
};

// byte offset of 16-byte chunk c of row r in a swizzled [rows][D] 16-bit tile
template <int D>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)(r * D * 2 + ((c ^ (r & 7)) << 4));
}

template <typename T, int D, bool PAGED, bool ROPE>
__global__ void __launch_bounds__(kThreads, D == 256 ? 1 : 2)
decode_tc_kernel(const Params p) {
  using C = TcCfg<D>;
  constexpr int DT = std::is_same<T, __half>::value ? B2_F16 : B2_BF16;
  extern __shared__ __align__(128) unsigned char smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sKV = sQ + C::kQBytes;  // stage s: K at sKV + 2s*tile, V after it
  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rep = p.Hq / p.Hkv;
  int lo, hi, qp;
  key_range(p, b, lo, hi, qp);
  const int s0 = lo + split * p.split_len, s1 = min(hi, s0 + p.split_len);
  const int ntiles = s1 > s0 ? (s1 - s0 + TK - 1) / TK : 0;

  // q rows (zero padded to 16) -> swizzled smem; plain stores, made visible
  // by the first __syncthreads of the main loop.
  for (int e = tid; e < 16 * C::kChunks; e += kThreads) {
    const int r = e / C::kChunks, c = e % C::kChunks;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (r < rep) val = *reinterpret_cast<const uint4*>((const T*)p.q + ((int64_t)b * p.Hq + hk * rep + r) * D + c * 8);
    if constexpr (ROPE) {  // rotate q at its position (4 pairs per chunk)
      uint32_t w[4] = {val.x, val.y, val.z, val.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float2 cs = rope_cs((double)qp, p.rope[c * 4 + u]);
        const float a = to_f32<T>(reinterpret_cast<const T*>(&w[u])[0]);
        const float d = to_f32<T>(reinterpret_cast<const T*>(&w[u])[1]);
        w[u] = pack2<T>(a * cs.x - d * cs.y, a * cs.y + d * cs.x);
      }
      val = make_uint4(w[0], w[1], w[2], w[3]);
    }
    *reinterpret_cast<uint4*>(smem + swz<D>(r, c)) = val;
  }

  const T* kb = (const T*)p.k;
  const T* vb = (const T*)p.v;
  const int cc = tid % C::kChunks, r0 = tid / C::kChunks;
  auto load_tile = [&](int t, int stage) {
    const int base = s0 + t * TK;
    const uint32_t dk = sKV + stage * 2 * C::kTileBytes, dv = dk + C::kTileBytes;
#pragma unroll
    for (int i = 0; i < TK / C::kRowsPerPass; ++i) {
      const int r = r0 + i * C::kRowsPerPass, pos = base + r;
      const bool ok = pos < s1;
      int64_t ko = 0, vo = 0;
      if (ok) {
        if constexpr (PAGED) {
          const int pg = p.page_table[(int64_t)b * p.max_pages + pos / p.page_size];
          const int off = pos - (pos / p.page_size) * p.page_size;
          ko = pg * p.ks[0] + off * p.ks[1] + hk * p.ks[2];
          vo = pg * p.vs[0] + off * p.vs[1] + hk * p.vs[2];
        } else {
          ko = b * p.ks[0] + hk * p.ks[1] + (int64_t)pos * p.ks[2];
          vo = b * p.vs[0] + hk * p.vs[1] + (int64_t)pos * p.vs[2];
        }
      }
      cp_async16_zfill(dk + swz<D>(r, cc), kb + ko + cc * 8, ok);
      cp_async16_zfill(dv + swz<D>(r, cc), vb + vo + cc * 8, ok);
    }
  };

#pragma unroll
  for (int st = 0; st < C::kStages - 1; ++st) {
    if (st < ntiles) load_tile(st, st);
    cp_async_commit_grp();
  }

  const float sl2 = p.scale * 1.4426950408889634f;  // scores in log2 units
  const int g = lane >> 2, tq = lane & 3;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // rows g, g + 8
  float acc[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;

  // per-lane ldmatrix row/chunk selectors
  const int qa_row = (lane & 7) + ((lane >> 3) & 1) * 8, qa_chunk = lane >> 4;
  const int kb_row = warp * 16 + (lane & 7) + ((lane >> 4) & 1) * 8, kb_chunk = (lane >> 3) & 1;
  const int vb_row = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, vb_chunk = lane >> 4;

  // RoPE on the staged keys: this thread rotates the chunks it loaded
  // (4 pairs of chunk cc, rows r0 + i * kRowsPerPass); the angle of the next
  // row is the previous one times the fixed step rotation.
  float2 rstep[4];
  if constexpr (ROPE) {
#pragma unroll
    for (int u = 0; u < 4; ++u) rstep[u] = rope_cs((double)C::kRowsPerPass, p.rope[cc * 4 + u]);
  }

  for (int t = 0; t < ntiles; ++t) {
    cp_async_wait_grp<C::kStages - 2>();
    __syncthreads();  // tile t visible to all; stage (t - 1) % S free
    {
      const int tn = t + C::kStages - 1;
      if (tn < ntiles) load_tile(tn, tn % C::kStages);
      cp_async_commit_grp();
    }
    const int stage = t % C::kStages;
    const uint32_t tk = sKV + stage * 2 * C::kTileBytes, tv = tk + C::kTileBytes;
    if constexpr (ROPE) {
      uint8_t* kt = smem + C::kQBytes + stage * 2 * C::kTileBytes;
      float2 cs[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) cs[u] = rope_cs((double)(s0 + t * TK + r0), p.rope[cc * 4 + u]);
#pragma unroll
      for (int i = 0; i < TK / C::kRowsPerPass; ++i) {
        uint4* ck = reinterpret_cast<uint4*>(kt + swz<D>(r0 + i * C::kRowsPerPass, cc));
        uint4 v4 = *ck;
        uint32_t w[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float a = to_f32<T>(reinterpret_cast<const T*>(&w[u])[0]);
          const float d = to_f32<T>(reinterpret_cast<const T*>(&w[u])[1]);
          w[u] = pack2<T>(a * cs[u].x - d * cs[u].y, a * cs[u].y + d * cs[u].x);
          const float2 nx = make_float2(cs[u].x * rstep[u].x - cs[u].y * rstep[u].y,
                                        cs[u].x * rstep[u].y + cs[u].y * rstep[u].x);
          cs[u] = nx;
        }
        *ck = make_uint4(w[0], w[1], w[2], w[3]);
      }
      __syncthreads();  // rotated keys visible to every warp
    }
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a[4], bk0[2], bk1[2];
      ldsm_x4(sQ + swz<D>(qa_row, 2 * kk + qa_chunk), a[0], a[1], a[2], a[3]);
      ldsm_x4(tk + swz<D>(kb_row, 2 * kk + kb_chunk), bk0[0], bk0[1], bk1[0], bk1[1]);
      mma_16816<DT>(s[0], a, bk0);
      mma_16816<DT>(s[1], a, bk1);
    }
    // scale, mask the ragged end, online softmax over this warp's 16 keys
    const int kpos = s0 + t * TK + warp * 16 + 2 * tq;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const bool ok = kpos + j * 8 + (e & 1) < s1;
        s[j][e] = ok ? s[j][e] * sl2 : -INFINITY;
      }
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float ref0 = mn0 == -INFINITY ? 0.f : mn0, ref1 = mn1 == -INFINITY ? 0.f : mn1;
    const float al0 = exp2f(m0 - ref0), al1 = exp2f(m1 - ref1);
    m0 = mn0;
    m1 = mn1;
    float pr[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      pr[j][0] = exp2f(s[j][0] - ref0);
      pr[j][1] = exp2f(s[j][1] - ref0);
      pr[j][2] = exp2f(s[j][2] - ref1);
      pr[j][3] = exp2f(s[j][3] - ref1);
    }
    l0 = l0 * al0 + (pr[0][0] + pr[0][1] + pr[1][0] + pr[1][1]);
    l1 = l1 * al1 + (pr[0][2] + pr[0][3] + pr[1][2] + pr[1][3]);
    uint32_t pa[4];
    pa[0] = pack2<T>(pr[0][0], pr[0][1]);
    pa[1] = pack2<T>(pr[0][2], pr[0][3]);
    pa[2] = pack2<T>(pr[1][0], pr[1][1]);
    pa[3] = pack2<T>(pr[1][2], pr[1][3]);
#pragma unroll
    for (int np = 0; np < D / 16; ++np) {
      uint32_t b0[2], b1[2];
      ldsm_x4_t(tv + swz<D>(vb_row, 2 * np + vb_chunk), b0[0], b0[1], b1[0], b1[1]);
      acc[2 * np][0] *= al0;
      acc[2 * np][1] *= al0;
      acc[2 * np][2] *= al1;
      acc[2 * np][3] *= al1;
      acc[2 * np + 1][0] *= al0;
      acc[2 * np + 1][1] *= al0;
      acc[2 * np + 1][2] *= al1;
      acc[2 * np + 1][3] *= al1;
      mma_16816<DT>(acc[2 * np], pa, b0);
      mma_16816<DT>(acc[2 * np + 1], pa, b1);
    }
  }
  cp_async_wait_grp<0>();
  __syncthreads();  // ring no longer read: reuse it for the merge

  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  float* sO = reinterpret_cast<float*>(smem + C::kQBytes);  // [warp][16][D]
  float* sM = sO + kWarps * 16 * D;                         // [warp][16]
  float* sL = sM + kWarps * 16;
  if (tq == 0) {
    sM[warp * 16 + g] = m0;
    sM[warp * 16 + g + 8] = m1;
    sL[warp * 16 + g] = l0;
    sL[warp * 16 + g + 8] = l1;
  }
#pragma unroll
  for (int n = 0; n < D / 8; ++n) {
    float* row0 = sO + (warp * 16 + g) * D + n * 8 + 2 * tq;
    float* row1 = row0 + 8 * D;
    *reinterpret_cast<float2*>(row0) = make_float2(acc[n][0], acc[n][1]);
    *reinterpret_cast<float2*>(row1) = make_float2(acc[n][2], acc[n][3]);
  }
  __syncthreads();
  for (int e = tid; e < rep * D; e += kThreads) {
    const int r = e / D, d = e % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sM[w * 16 + r]);
    const float ref = M == -INFINITY ? 0.f : M;
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float f = exp2f(sM[w * 16 + r] - ref);
      L += f * sL[w * 16 + r];
      O += f * sO[(w * 16 + r) * D + d];
    }
    const int hq = hk * rep + r;
    if (p.nsplit == 1) {
      ((T*)p.o)[((int64_t)b * p.Hq + hq) * D + d] = from_f32<T>(L > 0.f ? O / L : 0.f);
    } else {
      float* w = p.ws + (((int64_t)b * p.Hq + hq) * p.nsplit + split) * (D + 2);
      if (d == 0) {
        w[0] = M * 0.6931471805599453f;  // natural-log units, as the generic kernel
        w[1] = L;
      }
      w[2 + d] = O;
    }
  }
}

static size_t smem_bytes(int D) { return (size_t)(kMaxRep * D + 2 * TK * (D + 1) + kWarps * TK) * 4; }

// Splits: with at least one (batch, kv head) pair per SM a single split
// already keeps >= 2 x 32 KB of K/V in flight per SM, enough to saturate HBM,
// and avoids the partials round trip.  With fewer pairs the sequence is cut
// so that about 2 CTAs per SM run, each split at least 4 tiles long.
static int choose_splits(int B, int Hkv, int max_len) {
  const int pairs = B * Hkv;
  if (pairs >= num_sms()) return 1;
  int ns = (2 * num_sms() + pairs - 1) / pairs;
  const int max_ns = (max_len + 4 * TK - 1) / (4 * TK);
  if (ns > max_ns) ns = max_ns;
  return ns < 1 ? 1 : ns;
}

}  // namespace dec
}  // namespace b2

using namespace b2;

extern "C" size_t b2_decode_attn_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t max_seq_len) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || D <= 0) return 0;
  const int ns = dec::choose_splits((int)B, (int)Hkv, (int)max_seq_len);
  return (size_t)B * Hq * ns * (D + 2) * sizeof(float);
}

extern "C" int b2_decode_attn(const void* q, const void* k, const void* v, void* o, const int32_t* page_table,
                              const int32_t* seq_lens, void* workspace, int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                              int64_t max_seq_len, int64_t page_size, int64_t max_pages, const int64_t* k_strides,
                              const int64_t* v_strides, const int32_t* q_pos, int64_t window, const float* rope_freqs,
                              float scale, int q_dtype, int kv_dtype, void* stream) {
  B2_CHECK_ARG(q && k && v && o && seq_lens && k_strides && v_strides, B2_ERR_INVALID, "decode_attn: null pointer");
  B2_CHECK_ARG(B > 0 && Hq > 0 && Hkv > 0 && D > 0 && max_seq_len >= 0, B2_ERR_INVALID, "decode_attn: bad shape");
  B2_CHECK_ARG(Hq % Hkv == 0 && Hq / Hkv <= dec::kMaxRep, B2_ERR_UNSUPPORTED,
               "decode_attn: Hq/Hkv = %lld query heads per kv head (1..%d supported)", (long long)(Hq / Hkv),
               dec::kMaxRep);
  B2_CHECK_ARG(D <= dec::kMaxD, B2_ERR_UNSUPPORTED, "decode_attn: D=%lld > %d", (long long)D, dec::kMaxD);
  B2_CHECK_ARG(page_size == 0 || (page_table && page_size > 0 && max_pages > 0), B2_ERR_INVALID,
               "decode_attn: paged cache needs page_table, page_size, max_pages");
  B2_CHECK_ARG(page_size == 0 || max_seq_len <= page_size * max_pages, B2_ERR_INVALID,
               "decode_attn: max_seq_len %lld exceeds the page table's capacity %lld x %lld",
               (long long)max_seq_len, (long long)max_pages, (long long)page_size);
  B2_CHECK_ARG((q_dtype == B2_F32 || q_dtype == B2_F16 || q_dtype == B2_BF16) &&
                   (kv_dtype == B2_F32 || kv_dtype == B2_F16 || kv_dtype == B2_BF16),
               B2_ERR_DTYPE, "decode_attn: dtypes %d / %d", q_dtype, kv_dtype);
  dec::Params p;
  p.q = q;
  p.k = k;
  p.v = v;
  p.o = o;
  p.page_table = page_table;
  p.seq_lens = seq_lens;
  p.B = (int)B;
  p.Hq = (int)Hq;
  p.Hkv = (int)Hkv;
  p.D = (int)D;
  p.page_size = (int)page_size;
  p.max_pages = (int)max_pages;
  for (int i = 0; i < 3; ++i) {
    p.ks[i] = k_strides[i];
    p.vs[i] = v_strides[i];
  }
  p.scale = scale;
  p.q_pos = q_pos;
  p.window = (int)(window > 0 ? window : 0);
  p.cap = (int)max_seq_len;
  p.rope = rope_freqs;
  B2_CHECK_ARG(!rope_freqs || D % 2 == 0, B2_ERR_INVALID, "decode_attn: RoPE needs an even head dim");
  // with a window every sequence has at most `window` keys: split that
  const int64_t eff_len = (window > 0 && window < max_seq_len) ? window : max_seq_len;
  p.nsplit = dec::choose_splits(p.B, p.Hkv, (int)eff_len);
  p.split_len = (int)((eff_len + p.nsplit - 1) / p.nsplit);
  p.split_len = (p.split_len + dec::TK - 1) / dec::TK * dec::TK;
  if (p.split_len == 0) p.split_len = dec::TK;
  p.ws = (float*)workspace;
  B2_CHECK_ARG(p.nsplit == 1 || workspace, B2_ERR_INVALID, "decode_attn: workspace required (%d splits)", p.nsplit);
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 grid(p.nsplit, p.Hkv, p.B);
  // Tensor-core path: same 16-bit type for q and KV, D in {64, 128, 256},
  // 16-byte aligned rows (cp.async 16).
  const bool a16 = ((uintptr_t)k % 16 == 0) && ((uintptr_t)v % 16 == 0) && ((uintptr_t)q % 16 == 0);
  bool s16 = true;
  for (int i = 0; i < 3; ++i) s16 = s16 && p.ks[i] % 8 == 0 && p.vs[i] % 8 == 0;
  if (q_dtype == kv_dtype && q_dtype != B2_F32 && (D == 64 || D == 128 || D == 256) && a16 && s16) {
#define B2_TC2(T, DD, PG, RP)                                                                                \
  do {                                                                                                       \
    const int sm = dec::TcCfg<DD>::kSmem;                                                                    \
    set_max_smem((const void*)dec::decode_tc_kernel<T, DD, PG, RP>, sm);                                     \
    dec::decode_tc_kernel<T, DD, PG, RP><<<grid, dec::kThreads, sm, st>>>(p);                                \
  } while (0)
#define B2_TC(T, DD)                                    \
  do {                                                  \
    if (page_size) {                                    \
      if (rope_freqs) B2_TC2(T, DD, true, true);        \
      else B2_TC2(T, DD, true, false);                  \
    } else {                                            \
      if (rope_freqs) B2_TC2(T, DD, false, true);       \
      else B2_TC2(T, DD, false, false);                 \
    }                                                   \
  } while (0)
#define B2_TC_D(T)                 \
  do {                             \
    if (D == 64) B2_TC(T, 64);     \
    else if (D == 128) B2_TC(T, 128); \
    else B2_TC(T, 256);            \
  } while (0)
    if (q_dtype == B2_F16) {
      B2_TC_D(__half);
      if (p.nsplit > 1) dec::decode_combine_kernel<__half><<<p.B * p.Hq, 128, 0, st>>>(p);
    } else {
      B2_TC_D(__nv_bfloat16);
      if (p.nsplit > 1) dec::decode_combine_kernel<__nv_bfloat16><<<p.B * p.Hq, 128, 0, st>>>(p);
    }
#undef B2_TC_D
#undef B2_TC
#undef B2_TC2
    return launch_status("decode_attn");
  }
  const size_t smem = dec::smem_bytes(p.D);
#define B2_DEC(TQ, TKV)                                                                                     \
  do {                                                                                                      \
    if (page_size) {                                                                                        \
      set_max_smem((const void*)dec::decode_split_kernel<TQ, TKV, true>, (int)smem);                      \
      dec::decode_split_kernel<TQ, TKV, true><<<grid, dec::kThreads, smem, st>>>(p);                       \
    } else {                                                                                                \
      set_max_smem((const void*)dec::decode_split_kernel<TQ, TKV, false>, (int)smem);                     \
      dec::decode_split_kernel<TQ, TKV, false><<<grid, dec::kThreads, smem, st>>>(p);                      \
    }                                                                                                       \
    if (p.nsplit > 1) dec::decode_combine_kernel<TQ><<<p.B * p.Hq, 128, 0, st>>>(p);                        \
  } while (0)
#define B2_DEC_KV(TQ)                                              \
  do {                                                             \
    if (kv_dtype == B2_F32) B2_DEC(TQ, float);                     \
    else if (kv_dtype == B2_F16) B2_DEC(TQ, __half);               \
    else B2_DEC(TQ, __nv_bfloat16);                                \
  } while (0)
  if (q_dtype == B2_F32) B2_DEC_KV(float);
  else if (q_dtype == B2_F16) B2_DEC_KV(__half);
  else B2_DEC_KV(__nv_bfloat16);
#undef B2_DEC_KV
#undef B2_DEC
  return launch_status("decode_attn");
}

// ---------------------------------------------------------------------------
// repeat_kv (reference make_repeat_kv_kernel, _msl_templates.py:3434-3480):
//   out[h, s, d] = in[h / n_rep, s, d],  in [Hkv, S, D] -> out [Hkv n_rep, S, D].
// Each output head is one contiguous block of S * D elements copied from its
// kv head; 16-byte vectors when the block allows it (a pure HBM copy).
// ---------------------------------------------------------------------------
namespace b2 {
template <typename V>
__global__ void repeat_kv_kernel(const V* __restrict__ in, V* __restrict__ out, int64_t per_head, int64_t n_rep,
                                 int64_t total) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t h = i / per_head, w = i - h * per_head;
    out[i] = in[(h / n_rep) * per_head + w];
  }
}
}  // namespace b2

extern "C" int b2_repeat_kv(const void* input, void* output, int64_t n_kv_heads, int64_t seq_len, int64_t head_dim,
                            int64_t n_rep, int64_t elem_bytes, void* stream) {
  B2_CHECK_ARG(input && output, B2_ERR_INVALID, "repeat_kv: null pointer");
  B2_CHECK_ARG(n_kv_heads > 0 && seq_len >= 0 && head_dim > 0 && n_rep > 0, B2_ERR_INVALID, "repeat_kv: bad shape");
  B2_CHECK_ARG(elem_bytes == 1 || elem_bytes == 2 || elem_bytes == 4 || elem_bytes == 8, B2_ERR_DTYPE,
               "repeat_kv: element size %lld", (long long)elem_bytes);
  const int64_t bytes = seq_len * head_dim * elem_bytes;  // per head
  if (bytes == 0) return B2_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t nq = n_kv_heads * n_rep;
  const int grid = 4 * num_sms();
  if (bytes % 16 == 0 && aligned(input, 16) && aligned(output, 16)) {
    repeat_kv_kernel<uint4><<<grid, 256, 0, st>>>((const uint4*)input, (uint4*)output, bytes / 16, n_rep,
                                                  nq * (bytes / 16));
  } else if (bytes % 4 == 0 && aligned(input, 4) && aligned(output, 4)) {
    repeat_kv_kernel<uint32_t><<<grid, 256, 0, st>>>((const uint32_t*)input, (uint32_t*)output, bytes / 4, n_rep,
                                                     nq * (bytes / 4));
  } else {
    repeat_kv_kernel<uint8_t><<<grid, 256, 0, st>>>((const uint8_t*)input, (uint8_t*)output, bytes, n_rep,
                                                    nq * bytes);
  }
  return launch_status("repeat_kv");
}

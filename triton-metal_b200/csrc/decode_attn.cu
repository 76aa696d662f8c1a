// Decode attention (one query token per head) over a contiguous or paged KV
// cache, split-KV ("flash decoding"), sm_100a.
//
// Reference kernels this replaces (triton_metal/codegen/_msl_templates.py):
//   kv_cache_attention (:1949-2063), gqa_attention (:2064-2164),
//   batched_kv_decode (:2167-2278), paged_attention (:2279-2404),
//   multi_head_paged_attention (:2405-2532), fp16_kv_attention (:2533-2627).
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
#include "b2_common.cuh"

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
};

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
  const int len = p.seq_lens[b];
  const int s0 = split * p.split_len, s1 = min(len, s0 + p.split_len);

  for (int e = tid; e < rep * D; e += kThreads) {
    const int hh = e / D, d = e % D;
    sQ[e] = ldf((const TQ*)p.q + ((int64_t)b * p.Hq + hk * rep + hh) * D + d) * p.scale;
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

static size_t smem_bytes(int D) { return (size_t)(kMaxRep * D + 2 * TK * (D + 1) + kWarps * TK) * 4; }

// Splits so that B * Hkv * nsplit covers the SMs about twice, each split
// at least 4 tiles long.
static int choose_splits(int B, int Hkv, int max_len) {
  const int target = 2 * num_sms();
  int ns = (target + B * Hkv - 1) / (B * Hkv);
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
                              const int64_t* v_strides, float scale, int q_dtype, int kv_dtype, void* stream) {
  B2_CHECK_ARG(q && k && v && o && seq_lens && k_strides && v_strides, B2_ERR_INVALID, "decode_attn: null pointer");
  B2_CHECK_ARG(B > 0 && Hq > 0 && Hkv > 0 && D > 0 && max_seq_len >= 0, B2_ERR_INVALID, "decode_attn: bad shape");
  B2_CHECK_ARG(Hq % Hkv == 0 && Hq / Hkv <= dec::kMaxRep, B2_ERR_UNSUPPORTED,
               "decode_attn: Hq/Hkv = %lld query heads per kv head (1..%d supported)", (long long)(Hq / Hkv),
               dec::kMaxRep);
  B2_CHECK_ARG(D <= dec::kMaxD, B2_ERR_UNSUPPORTED, "decode_attn: D=%lld > %d", (long long)D, dec::kMaxD);
  B2_CHECK_ARG(page_size == 0 || (page_table && page_size > 0 && max_pages > 0), B2_ERR_INVALID,
               "decode_attn: paged cache needs page_table, page_size, max_pages");
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
  p.nsplit = dec::choose_splits(p.B, p.Hkv, (int)max_seq_len);
  p.split_len = (int)((max_seq_len + p.nsplit - 1) / p.nsplit);
  p.split_len = (p.split_len + dec::TK - 1) / dec::TK * dec::TK;
  if (p.split_len == 0) p.split_len = dec::TK;
  p.ws = (float*)workspace;
  B2_CHECK_ARG(p.nsplit == 1 || workspace, B2_ERR_INVALID, "decode_attn: workspace required (%d splits)", p.nsplit);
  cudaStream_t st = (cudaStream_t)stream;
  const size_t smem = dec::smem_bytes(p.D);
  const dim3 grid(p.nsplit, p.Hkv, p.B);
#define B2_DEC(TQ, TKV)                                                                                     \
  do {                                                                                                      \
    if (page_size) {                                                                                        \
      cudaFuncSetAttribute(dec::decode_split_kernel<TQ, TKV, true>,                                        \
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);                         \
      dec::decode_split_kernel<TQ, TKV, true><<<grid, dec::kThreads, smem, st>>>(p);                       \
    } else {                                                                                                \
      cudaFuncSetAttribute(dec::decode_split_kernel<TQ, TKV, false>,                                       \
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);                         \
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

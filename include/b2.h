/*
 * b2.h — C ABI of the B200-native (sm_100a) hot-path kernels.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * passed as void*.  Nothing here allocates device memory; the caller owns
 * every buffer, including the output (the convention of the reference's
 * Metal templates, where the caller binds every buffer by index:
 * triton_metal/codegen/_msl_templates.py:2705-2712 for INT4/INT8,
 * :1625-1630 for FlashAttention, :2086-2091 for GQA decode).
 *
 * Return value: B2_OK (0) or a negative B2_ERR_* code.  The message of the
 * last failure on the calling thread is returned by b2_last_error().
 * All launches are asynchronous on the given stream; no host sync inside.
 */
#ifndef B2_H_
#define B2_H_

#include <stdint.h>
#include <stddef.h>

#if defined(__GNUC__)
#define B2_API __attribute__((visibility("default")))
#else
#define B2_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define B2_OK               0
#define B2_ERR_INVALID    (-1)  /* bad shape / argument */
#define B2_ERR_DTYPE      (-2)  /* unsupported dtype combination */
#define B2_ERR_ALIGN      (-3)  /* pointer or stride alignment */
#define B2_ERR_UNSUPPORTED (-4) /* valid but not implemented shape */
#define B2_ERR_LAUNCH     (-5)  /* CUDA launch / runtime error */
#define B2_ERR_TIMEOUT    (-6)  /* a bounded device wait ran out */

/* dtype codes for activations / scales / outputs */
#define B2_F16  0
#define B2_BF16 1
#define B2_F32  2

/* int4 weight layouts */
#define B2_LAYOUT_GPTQ 0  /* int32 [K/8, N], nibble j of a word = k%8 == j   */
#define B2_LAYOUT_REF  1  /* uint8 [N, K/2], low nibble = even k (reference) */

B2_API int         b2_version(void);
B2_API const char* b2_last_error(void);
/* Synchronise `stream`, then read and clear the device error word that the
 * kernels' bounded waits set instead of hanging.  *code (may be NULL)
 * receives the raw code.  Returns B2_OK or B2_ERR_TIMEOUT.  Counterpart of
 * the reference's command-buffer status check
 * (triton_metal/backend/driver.py:218-225). */
B2_API int b2_device_error(void* stream, unsigned int* code);

/*
 * W4A16 group-wise weight-only matmul: output[M,N] = input[M,K] @ W
 * with W[k,n] = (q[k,n] - z[k/G,n]) * scales[k/G,n].
 * Replaces the reference kernel int4_matmul
 * (triton_metal/codegen/_msl_templates.py:2682-2745, buffer order
 * input, weight, output, scales, zeros, M, N, K at :2705-2712).
 *   weight  : B2_LAYOUT_GPTQ int32 [K/8, N]
 *   scales  : dtype [K/G, N]
 *   zeros   : NULL -> symmetric zero point 8 (the layout's default);
 *             else dtype [K/G, N] zero points (asymmetric).
 *   dtype   : B2_F16 or B2_BF16 for input, scales, zeros and output: the
 *             decode GEMV (M <= 16) or the tcgen05 prefill GEMM (M > 16);
 *             B2_F32 (the reference's own dtype) for input, scales, zeros
 *             and output: the reference's arithmetic, (q - z) * s and every
 *             product in fp32 on CUDA cores (K % 8 == 0, G % 8 == 0).
 */
B2_API int b2_int4_matmul(const void* input, const void* weight, void* output,
                   const void* scales, const void* zeros,
                   int64_t M, int64_t N, int64_t K, int64_t group_size,
                   int dtype, void* stream);

/*
 * W8A16 per-channel weight-only matmul: output[M,N] = input[M,K] @ W,
 * W[k,n] = (w8[n,k] - zeros[n]) * scales[n].
 * Replaces int8_matmul (triton_metal/codegen/_msl_templates.py:2630-2679,
 * buffer order input, weight, output, scales, zeros, M, N, K at :2652-2661).
 *   weight  : int8 [N, K] (K-major, the reference layout)
 *   scales  : dtype [N];  zeros: NULL (symmetric) or dtype [N].
 *   dtype   : B2_F16 / B2_BF16 (tensor cores), or B2_F32 (the reference's
 *             dtype: fp32 (w - z) * s and fp32 products, K % 8 == 0).
 */
B2_API int b2_int8_matmul(const void* input, const void* weight, void* output,
                   const void* scales, const void* zeros,
                   int64_t M, int64_t N, int64_t K,
                   int dtype, void* stream);

/*
 * int4_matmul in the reference's own buffers and layouts, natively
 * (make_int4_matmul_kernel, _msl_templates.py:2682-2745; buffer order
 * :2705-2712): weight uint8 [N, K/2], byte j of row n = k 2j (low nibble)
 * and 2j+1 (high nibble) (:2725-2732); scales and zeros [N, K/G] in the
 * activation dtype (zeros NULL = 8); input [M, K], output [M, N].
 * 16-bit dtypes: M <= 16: K-major mma.sync GEMV (K % 128 == 0, G % 32 ==
 * 0); M > 16: the tcgen05 prefill GEMM (K % 64 == 0, G % 64 == 0); else a
 * generic kernel.  B2_F32 (the reference's buffers as they are): fp32
 * scales / zeros / output and the reference's fp32 arithmetic.
 */
B2_API int b2_int4_matmul_ref(const void* input, const void* weight, void* output,
                              const void* scales, const void* zeros,
                              int64_t M, int64_t N, int64_t K, int64_t group_size,
                              int dtype, void* stream);

/*
 * Plain bf16 GEMM on tcgen05: out[M,N] = x[M,K] @ w[N,K]^T (w K-major, the
 * nn.Linear layout), fp32 accumulate, bf16 out.  The dequantised-weight
 * path of the reference's matmuls (x @ dequant(W), _msl_templates.py:2663,
 * :2716) when W is already bf16.  Any M; needs N % 8 == 0, K % 64 == 0
 * and 16-byte aligned pointers.
 */
B2_API int b2_gemm_bf16(const void* x, const void* w, void* out,
                        int64_t M, int64_t N, int64_t K, void* stream);

/*
 * Exact int4 -> fp32 dequantisation W[k,n] = (q - z) * float(s), written
 * as fp32 [K, N].  Debug/parity export of the unpack + dequant step the
 * reference does per k inside int4_matmul (_msl_templates.py:2723-2737).
 */
B2_API int b2_int4_dequant(const void* weight, const void* scales, const void* zeros,
                    float* out, int64_t N, int64_t K, int64_t group_size,
                    int dtype, void* stream);

/*
 * Repack the reference int4 layout uint8 [N, K/2] (low nibble = even k,
 * _msl_templates.py:2725-2732) into the GPTQ layout int32 [K/8, N].
 */
B2_API int b2_int4_repack_ref_to_gptq(const void* ref_weight, void* gptq_weight,
                               int64_t N, int64_t K, void* stream);

/*
 * Host plan of the W4 decode GEMV (M <= 16) for one shape; no device work.
 * info[6] = {grid, 8-column tiles per CTA slab, CTAs with one extra tile,
 * ring stages, quantisation groups per TMA box, shared-memory bytes} for a
 * GPU with `sms` SMs.  B2_ERR_UNSUPPORTED when the streaming GEMV does not
 * take the shape (b2_int4_matmul then runs the generic kernel).
 */
B2_API int b2_w4_gemv_plan(int64_t M, int64_t N, int64_t K, int64_t group_size, int zeros, int sms,
                           int64_t* info);

/*
 * FlashAttention forward.  q [B, Hq, S, D], k/v [B, Hkv, S, D], o like q,
 * each with arbitrary element strides (b, h, s; the last dim contiguous).
 * GQA maps q head h to kv head h / (Hq/Hkv), the reference's head map
 * (_msl_templates.py:2101-2104).  Replaces flash_attention
 * (_msl_templates.py:1568-1767, buffers Q, K, V, O, seq_len, scale) and the
 * strided Triton form _flash_attn_fwd (tests/test_flash_attention.py:24-104).
 *   dtype : B2_BF16 / B2_F16 (tcgen05 path) or B2_F32 (fp32 in/out).
 */
B2_API int b2_flash_attn_fwd(const void* q, const void* k, const void* v, void* o,
                      int64_t B, int64_t Hq, int64_t Hkv,
                      int64_t Sq, int64_t Skv, int64_t D,
                      const int64_t* q_strides, const int64_t* k_strides,
                      const int64_t* v_strides, const int64_t* o_strides,
                      float scale, int causal, int dtype, void* stream);

/*
 * Causal sliding-window FlashAttention (prefill): query s attends to keys
 * s - window + 1 .. s (window > 0; Sq == Skv).  Same tensors and strides as
 * b2_flash_attn_fwd; the prefill form of sliding_window_attention
 * (_msl_templates.py:3335-3431).  tcgen05 kernel for D = 128 bf16/fp16.
 */
B2_API int b2_flash_attn_fwd_window(const void* q, const void* k, const void* v, void* o,
                                    int64_t B, int64_t Hq, int64_t Hkv,
                                    int64_t Sq, int64_t Skv, int64_t D,
                                    const int64_t* q_strides, const int64_t* k_strides,
                                    const int64_t* v_strides, const int64_t* o_strides,
                                    float scale, int64_t window, int dtype, void* stream);

/*
 * Decode attention: one query token per head over a KV cache, split-KV.
 * Replaces kv_cache_attention, gqa_attention, batched_kv_decode,
 * paged_attention, multi_head_paged_attention and fp16_kv_attention
 * (triton_metal/codegen/_msl_templates.py:1949-2627).
 *   q [B, Hq, D] (q_dtype), o like q.
 *   page_size == 0: contiguous K/V [B, Hkv, S, D], k/v_strides = element
 *                   strides (b, h, s).
 *   page_size  > 0: paged K/V [n_pages, page_size, Hkv, D], page_table
 *                   int32 [B, max_pages] (logical -> physical page),
 *                   k/v_strides = element strides (page, token, head).
 *   seq_lens int32 [B] (<= max_seq_len); kv head of q head h = h / (Hq/Hkv).
 *   kv_dtype may differ from q_dtype (fp16 KV with fp32 queries).
 *   q_pos int32 [B] or NULL (= seq_len - 1): the query's position.
 *   window > 0: keys [max(0, q_pos + 1 - window), min(q_pos + 1, seq_len))
 *     (sliding_window_attention, _msl_templates.py:3335-3431); 0: [0, seq_len).
 *   rope_freqs fp32 [D/2] or NULL: rotate q at q_pos and key j at j, pairs
 *     (2d, 2d + 1) by pos * rope_freqs[d] (rope_attention, :1770-1887).
 *   workspace: b2_decode_attn_workspace_size(...) bytes (NULL when it is 0).
 */
B2_API size_t b2_decode_attn_workspace_size(int64_t B, int64_t Hq, int64_t Hkv,
                                            int64_t D, int64_t max_seq_len);
B2_API int b2_decode_attn(const void* q, const void* k, const void* v, void* o,
                          const int32_t* page_table, const int32_t* seq_lens,
                          void* workspace, int64_t B, int64_t Hq, int64_t Hkv,
                          int64_t D, int64_t max_seq_len, int64_t page_size,
                          int64_t max_pages, const int64_t* k_strides,
                          const int64_t* v_strides, const int32_t* q_pos,
                          int64_t window, const float* rope_freqs, float scale,
                          int q_dtype, int kv_dtype, void* stream);

/*
 * repeat_kv (make_repeat_kv_kernel, _msl_templates.py:3434-3480):
 *   out[h, s, d] = in[h / n_rep, s, d]; in [n_kv_heads, seq_len, head_dim],
 *   out [n_kv_heads * n_rep, seq_len, head_dim], elements of elem_bytes.
 */
B2_API int b2_repeat_kv(const void* input, void* output, int64_t n_kv_heads,
                        int64_t seq_len, int64_t head_dim, int64_t n_rep,
                        int64_t elem_bytes, void* stream);

/*
 * KDA (chunked gated delta rule) forward.  No reference counterpart: the
 * reference has no KDA code.  Layout [B, T, H, D] contiguous:
 *   q, k, v : dtype (B2_BF16) [B,T,H,Dk|Dv];  g : fp32 [B,T,H,Dk] log-decay
 *   beta    : dtype [B,T,H];  initial_state : fp32 [B,H,Dk,Dv] or NULL
 *   o       : dtype [B,T,H,Dv];  final_state : fp32 [B,H,Dk,Dv] or NULL
 *   workspace: device scratch of b2_kda_workspace_size(...) bytes
 *             (80,384 bytes per (b, h, 64-step chunk)), 16-byte aligned.
 * Two kernels: a per-chunk WY/UT transform on tcgen05 and the state +
 * output recurrence on clusters of two CTAs (one carries the state, its
 * partner computes the outputs); the state is carried in fp32.
 */
B2_API size_t b2_kda_workspace_size(int64_t B, int64_t T, int64_t H,
                             int64_t Dk, int64_t Dv, int64_t chunk);
B2_API int b2_kda_fwd(const void* q, const void* k, const void* v, const float* g,
               const void* beta, const float* initial_state,
               void* o, float* final_state, void* workspace,
               int64_t B, int64_t T, int64_t H, int64_t Dk, int64_t Dv,
               int64_t chunk, float scale, int dtype, void* stream);

/*
 * b2_kda_fwd without a workspace argument, for callers that cannot allocate
 * device memory when they run KDA (e.g. inside a custom allocator or memory
 * pool that must not be re-entered, or a plugin host that only provides the
 * input and output buffers).  No counterpart in the reference (which has no
 * KDA at all).  The workspace is a fixed 64 MiB device array inside the
 * library that every GPU loading it keeps until exit; shapes needing more
 * (B*H*(T/64) > 834 chunk-heads) are rejected with B2_ERR_INVALID.  The first call on a
 * device looks up the array's address (do it before any stream capture).
 * All calls share the array: calls overlapping on the GPU race.
 */
B2_API int b2_kda_fwd_noalloc(const void* q, const void* k, const void* v, const float* g,
                              const void* beta, const float* initial_state,
                              void* o, float* final_state,
                              int64_t B, int64_t T, int64_t H, int64_t Dk, int64_t Dv,
                              int64_t chunk, float scale, int dtype, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* B2_H_ */

"""Attention ops (torch tensors in, torch tensors out) backed by libb2.so.

  * flash_attention(q, k, v, causal, scale)  <- the strided Triton kernel
      _flash_attn_fwd (tests/test_flash_attention.py:24-104): q [B, Hq, S, D],
      k/v [B, Hkv, S, D] (any strides, last dim contiguous); GQA when
      Hkv < Hq with kv_head = q_head // (Hq // Hkv) (_msl_templates.py:2101).
  * flash_attention_template(Q, K, V, seq_len, scale, head_dim, causal)
      <- make_flash_attention_kernel's buffers (_msl_templates.py:1568-1630):
      Q/K/V/O [n_heads * seq_len, D].
  * gqa_attention(q, k_cache, v_cache, seq_len, scale, n_q_per_kv)
      <- make_gqa_attention_kernel's buffers (_msl_templates.py:2064-2091):
      q [n_q_heads, D], caches [n_kv_heads, seq_len, D] -> [n_q_heads, D].
D == 128 in bf16/fp16 runs the tcgen05 kernel; other shapes/dtypes run the
generic CUDA kernel.  There is no CPU path.
"""
import math

import torch

from . import _lib
from .errors import B2DtypeError, B2ShapeError

_DT = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}


def _stream():
    return _lib.current_stream()


def _strides(t):
    """(tensor with a contiguous last dim, its (b, h, s) element strides)."""
    if t.stride(3) != 1:
        t = t.contiguous()
    return t, _lib.strides_arg(t.stride()[:3])


def flash_attention(q, k, v, causal=False, scale=None, out=None, window=0):
    """O = softmax(scale Q K^T [causal]) V for [B, H, S, D] tensors (GQA when Hq > Hkv).

    window > 0 (needs causal): query s sees keys s - window + 1 .. s only
    (Mistral-style sliding window)."""
    for t in (q, k, v):
        if not t.is_cuda:
            raise B2ShapeError("b200kern ops take CUDA tensors (there is no CPU path)")
        if t.dim() != 4:
            raise B2ShapeError("flash_attention takes [B, H, S, D] tensors")
    if q.dtype not in _DT or k.dtype != q.dtype or v.dtype != q.dtype:
        raise B2DtypeError(f"q/k/v must share one of {list(_DT)}")
    B, Hq, Sq, D = q.shape
    Bk, Hkv, Skv, Dk = k.shape
    if Bk != B or Dk != D or tuple(v.shape) != tuple(k.shape):
        raise B2ShapeError("k/v must be [B, Hkv, Skv, D] matching q")
    if Hq % Hkv:
        raise B2ShapeError(f"Hq={Hq} must be a multiple of Hkv={Hkv}")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    o = (_lib.check_out(out, (B, Hq, Sq, D), q.dtype, "flash_attention", contiguous=False) if out is not None
         else torch.empty(B, Hq, Sq, D, dtype=q.dtype, device=q.device))
    q, qs = _strides(q)
    k, ks = _strides(k)
    v, vs = _strides(v)
    if o.stride(3) != 1:
        raise B2ShapeError("out must have a contiguous last dimension")
    os_ = _lib.strides_arg(o.stride()[:3])
    if window:
        if not causal or window < 0:
            raise B2ShapeError("a sliding window needs causal=True and window > 0")
        _lib.call("b2_flash_attn_fwd_window", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                  B, Hq, Hkv, Sq, Skv, D, qs, ks, vs, os_, float(scale), int(window), _DT[q.dtype], _stream())
        return o
    _lib.call("b2_flash_attn_fwd", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
              B, Hq, Hkv, Sq, Skv, D, qs, ks, vs, os_, float(scale), int(bool(causal)), _DT[q.dtype], _stream())
    return o


def flash_attention_template(Q, K, V, seq_len, scale, head_dim, causal=False):
    """Reference template buffers: [n_heads * seq_len, D] -> O of the same shape."""
    n = Q.numel() // (seq_len * head_dim)
    view = lambda t: t.reshape(1, n, seq_len, head_dim)
    return flash_attention(view(Q), view(K), view(V), causal=causal, scale=scale).reshape(-1, head_dim)


def gqa_attention(q, k_cache, v_cache, seq_len, scale, n_q_per_kv):
    """Decode attention: one query per q head over the KV cache of head q // n_q_per_kv."""
    hq, d = q.shape
    hkv = k_cache.numel() // (seq_len * d)
    if hq != hkv * n_q_per_kv:
        raise B2ShapeError(f"{hq} q heads != {hkv} kv heads x {n_q_per_kv}")
    kk = k_cache.reshape(1, hkv, seq_len, d)
    vv = v_cache.reshape(1, hkv, seq_len, d)
    return decode_attention(q.reshape(1, hq, d), kk, vv, seq_len, scale).reshape(hq, d)


# --------------------------------------------------------------------------
# decode attention over a KV cache (one query token per head)
# --------------------------------------------------------------------------
def _seq_lens(seq_lens, B, device):
    """int, sequence or tensor of B per-sequence integers -> int32 [B] on device."""
    if isinstance(seq_lens, int):
        return torch.full((B,), seq_lens, dtype=torch.int32, device=device)
    t = torch.as_tensor(seq_lens).to(device=device, dtype=torch.int32).reshape(-1).contiguous()
    if t.numel() != B:
        raise B2ShapeError(f"expected {B} per-sequence values, got {t.numel()}")
    return t


def decode_attention(q, k_cache, v_cache, seq_lens, scale=None, page_table=None, out=None, q_pos=None, window=0,
                     rope_freqs=None):
    """o[B, Hq, D] = softmax(scale q K^T) V over the first seq_lens[b] keys.

    Contiguous cache: k/v [B, Hkv, S, D] (any strides, last dim contiguous).
    Paged cache (page_table int32 [B, max_pages] given): k/v
    [n_pages, page_size, Hkv, D].  GQA: kv head = q head // (Hq // Hkv).
    The cache dtype may differ from q's (e.g. fp16 KV with fp32 queries).
    q_pos [B] (default seq_len - 1); window > 0 keeps the keys
    [max(0, q_pos + 1 - window), min(q_pos + 1, seq_len)) (sliding window);
    rope_freqs [D/2] rotates q at q_pos and each key at its position (RoPE)."""
    for t in (q, k_cache, v_cache):
        if not t.is_cuda:
            raise B2ShapeError("b200kern ops take CUDA tensors (there is no CPU path)")
    if q.dim() != 3:
        raise B2ShapeError("q must be [B, Hq, D]")
    if q.dtype not in _DT or k_cache.dtype not in _DT or v_cache.dtype != k_cache.dtype:
        raise B2DtypeError("q and the cache must be fp32, fp16 or bf16")
    B, Hq, D = q.shape
    if k_cache.stride(-1) != 1:
        k_cache = k_cache.contiguous()
    if v_cache.stride(-1) != 1:
        v_cache = v_cache.contiguous()
    if page_table is None:
        Hkv, S = k_cache.shape[1], k_cache.shape[2]
        ks, vs = k_cache.stride()[:3], v_cache.stride()[:3]
        ps, max_pages, pt = 0, 0, None
    else:
        ps, Hkv = k_cache.shape[1], k_cache.shape[2]
        pt = page_table.to(device=q.device, dtype=torch.int32).contiguous()
        max_pages = pt.shape[1]
        S = max_pages * ps
        ks, vs = k_cache.stride()[:3], v_cache.stride()[:3]
    if Hq % Hkv:
        raise B2ShapeError(f"Hq={Hq} must be a multiple of Hkv={Hkv}")
    lens = _seq_lens(seq_lens, B, q.device)
    scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    q = q.contiguous()
    o = (_lib.check_out(out, (B, Hq, D), q.dtype, "decode_attention") if out is not None
         else torch.empty(B, Hq, D, dtype=q.dtype, device=q.device))
    lib = _lib.load()
    need = int(lib.b2_decode_attn_workspace_size(B, Hq, Hkv, D, S))
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
    qp = None if q_pos is None else _seq_lens(q_pos, B, q.device)
    fr = None
    if rope_freqs is not None:
        fr = torch.as_tensor(rope_freqs, dtype=torch.float32).to(q.device).contiguous()
        if fr.numel() != D // 2:
            raise B2ShapeError(f"rope_freqs must have D/2 = {D // 2} entries")
    _lib.call("b2_decode_attn", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), o.data_ptr(),
              None if pt is None else pt.data_ptr(), lens.data_ptr(), ws.data_ptr(), B, Hq, Hkv, D, S, ps,
              max_pages, _lib.strides_arg(ks), _lib.strides_arg(vs), None if qp is None else qp.data_ptr(),
              int(window), None if fr is None else fr.data_ptr(), scale, _DT[q.dtype], _DT[k_cache.dtype],
              _stream())
    return o


def sliding_window_attention(Q, K_cache, V_cache, q_pos, seq_len, window_size, scale=None):
    """Reference sliding_window_attention (_msl_templates.py:3335-3431):
    Q [D] (or [H, D]), caches [S, D] (or [H, S, D]); keys
    [max(0, q_pos + 1 - window_size), min(q_pos + 1, seq_len))."""
    D = Q.shape[-1]
    Qh = Q.reshape(1, -1, D)
    H = Qh.shape[1]
    K = K_cache.reshape(1, H, -1, D)
    V = V_cache.reshape(1, H, -1, D)
    return decode_attention(Qh, K, V, seq_len, scale, q_pos=[int(q_pos)], window=int(window_size)).reshape(Q.shape)


def rope_attention(Q, K_cache, V_cache, freqs, seq_len, q_pos):
    """Reference rope_attention (_msl_templates.py:1770-1887): Q [D] rotated at
    q_pos, un-rotated caches [S, D] rotated at each key's position, freqs
    [D/2], scale 1/sqrt(D), keys [0, seq_len)."""
    D = Q.shape[-1]
    Qh = Q.reshape(1, -1, D)
    H = Qh.shape[1]
    K = K_cache.reshape(1, H, -1, D)
    V = V_cache.reshape(1, H, -1, D)
    return decode_attention(Qh, K, V, seq_len, q_pos=[int(q_pos)], rope_freqs=freqs).reshape(Q.shape)


def repeat_kv(x, n_rep, out=None):
    """Reference repeat_kv (_msl_templates.py:3434-3480): [Hkv, S, D] ->
    [Hkv * n_rep, S, D] with out[h] = x[h // n_rep] (any leading batch dims
    folded: [..., Hkv, S, D] -> [..., Hkv * n_rep, S, D])."""
    if not x.is_cuda:
        raise B2ShapeError("b200kern ops take CUDA tensors (there is no CPU path)")
    if x.dim() < 3:
        raise B2ShapeError("repeat_kv takes [..., Hkv, S, D]")
    x = x.contiguous()
    *lead, Hkv, S, D = x.shape
    nb = 1
    for d in lead:
        nb *= d
    res = (_lib.check_out(out, (*lead, Hkv * n_rep, S, D), x.dtype, "repeat_kv") if out is not None
           else torch.empty(*lead, Hkv * n_rep, S, D, dtype=x.dtype, device=x.device))
    _lib.call("b2_repeat_kv", x.data_ptr(), res.data_ptr(), nb * Hkv, S, D, int(n_rep), x.element_size(), _stream())
    return res


def kv_cache_attention(Q, K_cache, V_cache, seq_len, scale):
    """Reference kv_cache_attention buffers: Q [H, D], caches [H, max_seq, D]."""
    H, D = Q.shape
    K = K_cache.reshape(1, H, -1, D)
    V = V_cache.reshape(1, H, -1, D)
    return decode_attention(Q.reshape(1, H, D), K, V, seq_len, scale).reshape(H, D)


def batched_kv_decode(Q, K_cache, V_cache, seq_lens, max_seq_len):
    """Reference batched_kv_decode: Q [B, H, D], caches [B, H, max_seq_len, D]."""
    B, H, D = Q.shape
    K = K_cache.reshape(B, H, max_seq_len, D)
    V = V_cache.reshape(B, H, max_seq_len, D)
    return decode_attention(Q, K, V, seq_lens)


def paged_attention(Q, K_pages, V_pages, page_table, seq_len, n_pages, page_size):
    """Reference paged_attention (one head: K_pages [P, page_size, D]) and
    multi_head_paged_attention (Q [H, D], K_pages [P, page_size, H, D])."""
    D = Q.shape[-1]
    Qh = Q.reshape(1, -1, D)
    H = Qh.shape[1]
    K = K_pages.reshape(-1, page_size, H, D)
    V = V_pages.reshape(-1, page_size, H, D)
    pt = page_table.reshape(1, -1)[:, :n_pages]
    return decode_attention(Qh, K, V, seq_len, page_table=pt).reshape(Q.shape)

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
    return torch.cuda.current_stream().cuda_stream


def _strides(t):
    """(tensor with a contiguous last dim, its (b, h, s) element strides)."""
    if t.stride(3) != 1:
        t = t.contiguous()
    return t, _lib.strides_arg(t.stride()[:3])


def flash_attention(q, k, v, causal=False, scale=None, out=None):
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
    o = out if out is not None else torch.empty(B, Hq, Sq, D, dtype=q.dtype, device=q.device)
    q, qs = _strides(q)
    k, ks = _strides(k)
    v, vs = _strides(v)
    if o.stride(3) != 1:
        raise B2ShapeError("out must have a contiguous last dimension")
    os_ = _lib.strides_arg(o.stride()[:3])
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
    qq = q.reshape(1, hq, 1, d)
    kk = k_cache.reshape(1, hkv, seq_len, d)
    vv = v_cache.reshape(1, hkv, seq_len, d)
    return flash_attention(qq, kk, vv, causal=False, scale=scale).reshape(hq, d)

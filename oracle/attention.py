"""CPU oracle for attention (numpy, float64).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm as the checker.  Never the product.

Restates the reference's attention math:
  * _ref_attention (tests/test_flash_attention.py:107-118): scale 1/sqrt(D),
    S = (q*scale) @ k^T, causal mask tril (key <= query) filled with -inf,
    softmax over keys, NaN (all-masked rows) -> 0, O = P @ V.
  * flash_attention template (_msl_templates.py:1697-1753): the same result
    via online softmax; buffers [n_heads*seq_len, D] head-major.
  * GQA head map kv_head = q_head / n_q_per_kv (_msl_templates.py:2101-2104).
"""
import numpy as np


def attention(q, k, v, causal=False, scale=None):
    """q [..., Hq, Sq, D], k/v [..., Hkv, Skv, D] -> [..., Hq, Sq, D] float64.

    Causal follows the reference mask: key j is visible to query i iff j <= i
    (tests/test_flash_attention.py:111-114 builds tril over an N x N square).
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    hq, hkv = q.shape[-3], k.shape[-3]
    if hq != hkv:
        rep = hq // hkv
        k = np.repeat(k, rep, axis=-3)
        v = np.repeat(v, rep, axis=-3)
    if scale is None:
        scale = 1.0 / np.sqrt(q.shape[-1])
    s = (q * scale) @ np.swapaxes(k, -1, -2)
    if causal:
        sq, skv = s.shape[-2], s.shape[-1]
        mask = np.tril(np.ones((sq, skv), dtype=bool))
        s = np.where(mask, s, -np.inf)
    m = np.max(s, axis=-1, keepdims=True)
    with np.errstate(invalid="ignore"):
        p = np.exp(s - m)
        p = p / np.sum(p, axis=-1, keepdims=True)
    p = np.nan_to_num(p, nan=0.0)
    return p @ v


def flash_attention_template(Q, K, V, seq_len, scale, head_dim, causal=False):
    """The reference template's buffers: Q/K/V [n_heads*seq_len, D] -> O."""
    Q = np.asarray(Q, dtype=np.float64).reshape(-1, seq_len, head_dim)
    K = np.asarray(K, dtype=np.float64).reshape(-1, seq_len, head_dim)
    V = np.asarray(V, dtype=np.float64).reshape(-1, seq_len, head_dim)
    return attention(Q, K, V, causal=causal, scale=scale).reshape(-1, head_dim)


def gqa_decode(q, k_cache, v_cache, seq_len, scale, n_q_per_kv):
    """Reference gqa_attention buffers: q [Hq, D], caches [Hkv, S, D] -> [Hq, D]."""
    q = np.asarray(q, dtype=np.float64)
    hq, d = q.shape
    kc = np.asarray(k_cache, dtype=np.float64).reshape(-1, seq_len, d)
    vc = np.asarray(v_cache, dtype=np.float64).reshape(-1, seq_len, d)
    out = np.empty((hq, d))
    for h in range(hq):
        kv = h // n_q_per_kv
        s = kc[kv] @ q[h] * scale
        p = np.exp(s - s.max())
        out[h] = (p / p.sum()) @ vc[kv]
    return out

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
  * sliding window decode (_msl_templates.py:3335-3431): keys
    [max(0, q_pos + 1 - W), min(q_pos + 1, seq_len)).
  * fused RoPE decode (_msl_templates.py:1770-1887): q rotated at q_pos, key
    j at position j, pairs (2d, 2d + 1) with angle pos * freqs[d]; V is not
    rotated; keys [0, seq_len); scale 1/sqrt(D).
  * repeat_kv (_msl_templates.py:3434-3480): out[h, s, d] = in[h // n_rep, s, d].
"""
import numpy as np


def attention(q, k, v, causal=False, scale=None, window=0):
    """q [..., Hq, Sq, D], k/v [..., Hkv, Skv, D] -> [..., Hq, Sq, D] float64.

    Causal follows the reference mask: key j is visible to query i iff j <= i
    (tests/test_flash_attention.py:111-114 builds tril over an N x N square).
    window > 0 (with causal) also hides keys j <= i - window: the key range
    the reference's sliding_window_attention keeps for a query at position i
    (_msl_templates.py:3335-3431, start = max(0, pos + 1 - window)).
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
        if window > 0:
            mask &= ~np.tril(np.ones((sq, skv), dtype=bool), -window)
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


def rope_rotate(x, pos, freqs):
    """Rotate pairs (2d, 2d + 1) of x [..., D] by angle pos * freqs[d]
    (_msl_templates.py:1817-1825 for q, :1836-1842 for each key)."""
    x = np.asarray(x, dtype=np.float64)
    th = np.multiply.outer(np.asarray(pos, dtype=np.float64), np.asarray(freqs, dtype=np.float64))
    c, s = np.cos(th), np.sin(th)
    xr, xi = x[..., 0::2], x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = xr * c - xi * s
    out[..., 1::2] = xr * s + xi * c
    return out


def decode(q, k_cache, v_cache, seq_lens, scale=None, q_pos=None, window=0, rope_freqs=None):
    """Single-token decode attention, float64.

    q [B, Hq, D]; k/v [B, Hkv, S, D] (S >= every seq_len); seq_lens [B].
    kv head of q head h is h // (Hq // Hkv) (_msl_templates.py:2101-2104);
    keys beyond seq_len are ignored (kv-cache templates, :1949-2063,
    :2167-2278); an empty key range gives 0 (the nan_to_num convention of
    tests/test_flash_attention.py:117).
    q_pos [B] (default seq_len - 1) is the query's position.  window > 0
    keeps keys [max(0, q_pos + 1 - window), min(q_pos + 1, seq_len))
    (sliding window, :3372-3374).  rope_freqs [D/2] rotates q at q_pos and
    key j at j before the dot products (fused RoPE, :1770-1887).
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k_cache, dtype=np.float64)
    v = np.asarray(v_cache, dtype=np.float64)
    B, Hq, D = q.shape
    rep = Hq // k.shape[1]
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    out = np.zeros((B, Hq, D))
    for b in range(B):
        n = int(seq_lens[b])
        qp = n - 1 if q_pos is None else int(q_pos[b])
        lo, hi = 0, n
        if window > 0:
            lo, hi = max(0, qp + 1 - window), min(qp + 1, n)
        if hi <= lo:
            continue
        kb = k[b, :, lo:hi]
        qb = q[b]
        if rope_freqs is not None:
            kb = rope_rotate(kb, np.arange(lo, hi), rope_freqs)
            qb = rope_rotate(qb, qp, rope_freqs)
        for h in range(Hq):
            s = kb[h // rep] @ qb[h] * scale
            p = np.exp(s - s.max())
            out[b, h] = (p / p.sum()) @ v[b, h // rep, lo:hi]
    return out


def sliding_window_decode(q, k_cache, v_cache, q_pos, seq_len, window, scale=None):
    """Reference sliding_window_attention buffers: q [D], caches [S, D] -> [D]."""
    q = np.asarray(q, dtype=np.float64)
    d = q.shape[-1]
    kc = np.asarray(k_cache, dtype=np.float64).reshape(-1, d)
    vc = np.asarray(v_cache, dtype=np.float64).reshape(-1, d)
    return decode(q.reshape(1, 1, d), kc[None, None], vc[None, None], [seq_len], scale,
                  q_pos=[q_pos], window=window)[0, 0]


def rope_decode(q, k_cache, v_cache, freqs, seq_len, q_pos):
    """Reference rope_attention buffers: q [D], caches [S, D], freqs [D/2] -> [D]."""
    q = np.asarray(q, dtype=np.float64)
    d = q.shape[-1]
    kc = np.asarray(k_cache, dtype=np.float64).reshape(-1, d)
    vc = np.asarray(v_cache, dtype=np.float64).reshape(-1, d)
    return decode(q.reshape(1, 1, d), kc[None, None], vc[None, None], [seq_len], None,
                  q_pos=[q_pos], rope_freqs=freqs)[0, 0]


def repeat_kv(x, n_rep):
    """[Hkv, S, D] -> [Hkv * n_rep, S, D], out[h] = x[h // n_rep]."""
    return np.repeat(np.asarray(x), n_rep, axis=0)


def gather_pages(pages, page_table, seq_len):
    """Paged KV [n_phys_pages, page_size, (H,) D] + logical->physical table ->
    contiguous [seq_len, (H,) D] (_msl_templates.py:2279-2532)."""
    pages = np.asarray(pages)
    ps = pages.shape[1]
    rows = [pages[int(page_table[t // ps]), t % ps] for t in range(seq_len)]
    return np.stack(rows) if rows else np.zeros((0,) + pages.shape[2:])

"""CPU oracle for the KDA chunked gated-delta-rule forward (numpy float64).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm as the checker.  Never the product.

The reference (triton-metal) has no KDA code, so there is nothing in it to
pin this against.  The arithmetic's third-party home is flash-linear-attention
0.5.1 (fla.ops.kda.naive.naive_recurrent_kda); this module restates the
published recurrence and tests/golden/make_golden.py pins it against that
library's outputs (fixtures kda_*.npz).  Per head, with state S [Dk, Dv]:
  S <- S * exp(g_t)[:, None]
  u_t = v_t - S^T k_t
  S <- S + beta_t k_t u_t^T
  o_t = S^T (scale * q_t)
"""
import numpy as np


def recurrent(q, k, v, g, beta, scale=None, initial_state=None):
    """q, k, g [B, T, H, Dk]; v [B, T, H, Dv]; beta [B, T, H] -> (o [B,T,H,Dv], S [B,H,Dk,Dv])."""
    q, k, v, g, beta = (np.asarray(a, dtype=np.float64) for a in (q, k, v, g, beta))
    B, T, H, Dk = q.shape
    Dv = v.shape[-1]
    scale = Dk ** -0.5 if scale is None else scale
    S = np.zeros((B, H, Dk, Dv)) if initial_state is None else np.array(initial_state, dtype=np.float64)
    o = np.zeros((B, T, H, Dv))
    for t in range(T):
        S = S * np.exp(g[:, t])[..., None]
        kt = k[:, t]
        u = v[:, t] - np.einsum("bhk,bhkv->bhv", kt, S)
        S = S + np.einsum("bhk,bhv->bhkv", beta[:, t][..., None] * kt, u)
        o[:, t] = np.einsum("bhk,bhkv->bhv", q[:, t] * scale, S)
    return o, S


def make_inputs(B, T, H, D, seed=0):
    """BASELINE C4 distributions: q, k ~ N(0,1) then L2-normalised over D;
    v ~ N(0,1); g = -softplus(N(0,1)); beta = sigmoid(N(0,1))."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, T, H, D))
    k = rng.standard_normal((B, T, H, D))
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((B, T, H, D))
    g = -np.log1p(np.exp(rng.standard_normal((B, T, H, D))))
    beta = 1.0 / (1.0 + np.exp(-rng.standard_normal((B, T, H))))
    return q, k, v, g, beta

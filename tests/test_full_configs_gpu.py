"""Parity at the BASELINE configs' full sizes, through the public ops (C ABI).

Each test runs the whole problem on the GPU and checks a deterministic
sample of it against the float64 CPU oracle:

* C3 FlashAttention GQA prefill (B=4, Hq=32, Hkv=8, S=8192, D=128, causal,
  bf16, q/k/v = 0.5 N(0,1)): four (b, h) pairs, including the last batch and
  the last head; in each, the first, a middle and the last 128-row Q tile.
  |x - ref| <= 1e-2 + 1e-2 |ref| (north star rtol / atol).
* C2 W4A16 / C2' W8A16 prefill GEMMs (4096 x 4096 x 14336): three whole
  256-row CTA tiles (the first, a middle and the last), every column, so both
  128-row TMEM accumulator halves, all four epilogue warps and every N tile
  are compared.  W4 uses the RMS-scaled bound of the rounded dequantised
  operand, |x - ref| <= 1e-2 (|ref| + rms(ref)); W8 (integer weights exact
  in bf16) the plain 1e-2 bound.
* C4 KDA (B=1, H=32, T=16384): the final state at T = 16384 and every output
  step of two heads vs the float64 recurrence at 2e-2 (north star).

Mirrors the reference's seeded, shape-parameterised checks
(tests/test_flash_attention.py:144-188).
"""
import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import kda as okda
from oracle import quant as oq

pytestmark = pytest.mark.gpu


def _assert_within(err, bound, what):
    ok = err <= bound
    assert bool(ok.all()), (f"{what}: {int((~ok).sum())} elements out of tolerance, max err {float(err.max()):.4g}, "
                            f"worst ratio {float((err / bound).max()):.3g}")


def test_c3_fa_gqa_full_config(cuda):
    import b200kern as bk
    B, Hq, Hkv, S, D = 4, 32, 8, 8192, 128
    g = torch.Generator().manual_seed(0)
    q = (torch.randn(B, Hq, S, D, generator=g) * 0.5).bfloat16()
    k = (torch.randn(B, Hkv, S, D, generator=g) * 0.5).bfloat16()
    v = (torch.randn(B, Hkv, S, D, generator=g) * 0.5).bfloat16()
    o = bk.flash_attention(q.to(cuda), k.to(cuda), v.to(cuda), causal=True)
    torch.cuda.synchronize()
    assert o.shape == (B, Hq, S, D) and o.dtype == torch.bfloat16
    rows = np.concatenate([np.arange(0, 128), np.arange(4096 - 64, 4096 + 64), np.arange(S - 128, S)])
    rep = Hq // Hkv
    for (b, h) in ((0, 0), (1, 13), (2, 22), (B - 1, Hq - 1)):
        qr = q[b, h, rows].double().numpy()
        kk = k[b, h // rep].double().numpy()
        vv = v[b, h // rep].double().numpy()
        s = (qr / np.sqrt(D)) @ kk.T
        s = np.where(np.arange(S)[None, :] <= rows[:, None], s, -np.inf)
        p = np.exp(s - s.max(-1, keepdims=True))
        ref = (p / p.sum(-1, keepdims=True)) @ vv
        got = o[b, h, torch.from_numpy(rows)].double().cpu().numpy()
        err = np.abs(got - ref)
        _assert_within(err, 1e-2 + 1e-2 * np.abs(ref), f"C3 (b={b}, h={h})")
    # the oracle module itself on one small slice of the same tensors
    ref0 = oatt.attention(q[0, :1, :256].double().numpy(), k[0, :1, :256].double().numpy(),
                          v[0, :1, :256].double().numpy(), causal=True)
    got0 = o[0, :1, :256].double().cpu().numpy()
    _assert_within(np.abs(got0 - ref0), 1e-2 + 1e-2 * np.abs(ref0), "C3 oracle slice")


C2_TILES = [np.arange(0, 256), np.arange(2048, 2304), np.arange(4096 - 256, 4096)]


def test_c2_w4a16_gemm_whole_tiles(cuda):
    import b200kern as bk
    from b200kern.synthetic import w4_inputs
    d = w4_inputs(4096, 14336, 4096, group_size=128, dtype=torch.bfloat16, seed=0)
    out = bk.int4_matmul(d["x"].to(cuda), d["qweight"].to(cuda), d["scales"].to(cuda))
    torch.cuda.synchronize()
    rows = np.concatenate(C2_TILES)
    ref = oq.int4_matmul(d["x"][torch.from_numpy(rows)].double().numpy(), d["q"].numpy(),
                         d["scales"].double().numpy(), None, 128)
    got = out[torch.from_numpy(rows)].double().cpu().numpy()
    rms = np.sqrt((ref ** 2).mean())
    _assert_within(np.abs(got - ref), 1e-2 * (np.abs(ref) + rms), "C2 W4A16")


def test_c2_w8a16_gemm_whole_tiles(cuda):
    import b200kern as bk
    from b200kern.synthetic import w8_inputs
    d = w8_inputs(4096, 14336, 4096, dtype=torch.bfloat16, seed=0)
    out = bk.int8_matmul(d["x"].to(cuda), d["w"].to(cuda), d["scales"].to(cuda))
    torch.cuda.synchronize()
    rows = np.concatenate(C2_TILES)
    ref = oq.int8_matmul(d["x"][torch.from_numpy(rows)].double().numpy(), d["w"].numpy(),
                         d["scales"].double().numpy())
    got = out[torch.from_numpy(rows)].double().cpu().numpy()
    _assert_within(np.abs(got - ref), 1e-2 + 1e-2 * np.abs(ref), "C2' W8A16")


def test_c4_kda_final_state_and_outputs(cuda):
    import b200kern as bk
    B, T, H, D = 1, 16384, 32, 128
    gen = torch.Generator().manual_seed(0)
    F = torch.nn.functional
    q = F.normalize(torch.randn(B, T, H, D, generator=gen), dim=-1).bfloat16()
    k = F.normalize(torch.randn(B, T, H, D, generator=gen), dim=-1).bfloat16()
    v = torch.randn(B, T, H, D, generator=gen).bfloat16()
    g = -F.softplus(torch.randn(B, T, H, D, generator=gen))
    beta = torch.sigmoid(torch.randn(B, T, H, generator=gen)).bfloat16()
    o, S = bk.kda_chunk_fwd(q.to(cuda), k.to(cuda), v.to(cuda), g.to(cuda), beta.to(cuda))
    torch.cuda.synchronize()
    heads = [0, H - 1]
    sel = lambda t: t[:, :, heads].double().numpy()
    oref, Sref = okda.recurrent(sel(q), sel(k), sel(v), sel(g), beta[:, :, heads].double().numpy())
    got_o = o[:, :, heads].double().cpu().numpy()
    got_s = S[:, heads].double().cpu().numpy()
    tol = 2e-2
    _assert_within(np.abs(got_s - Sref), tol + tol * np.abs(Sref), "C4 final state")
    _assert_within(np.abs(got_o - oref), tol + tol * np.abs(oref), "C4 outputs")

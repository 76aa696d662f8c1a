"""Parity of the FlashAttention kernels (through the C ABI) with the oracle.

Tolerances: the reference's own fp32 tests use max abs error < 0.01
(tests/test_flash_attention.py:155, :188); bf16/fp16 paths are checked
against an fp32 reference of the same rounded inputs with
|out - ref| <= 1e-2 + 1e-2 |ref| (the north-star rtol/atol)."""
import json
import math
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden
from oracle import attention as oatt

pytestmark = pytest.mark.gpu
MANIFEST = json.load(open(os.path.join(GOLDEN, "manifest.json")))
REF_TESTS = {r["test"]: r for r in MANIFEST["reference_tests"]}


def _close(out, ref, tol=1e-2):
    out, ref = out.float(), ref.float()
    err = (out - ref).abs()
    bound = tol + tol * ref.abs()
    assert bool((err <= bound).all()), f"max err {err.max().item():.4g}, ratio {(err / bound).max().item():.3g}"


@pytest.mark.parametrize("rec", MANIFEST["triton_fa"], ids=lambda r: r["name"])
def test_triton_fa_golden(cuda, rec):
    """The reference's strided Triton test cases (seed 42, fp32) vs _ref_attention."""
    import b200kern as bk
    g = golden(rec["name"])
    q, k, v = (torch.tensor(g[n], device=cuda) for n in "qkv")
    out = bk.flash_attention(q, k, v, causal=rec["causal"])
    assert (out.cpu() - torch.tensor(g["out"])).abs().max().item() < 0.01


# Each reference test's own acceptance rule, |got - expected| < max(atol, rtol |expected|)
# (tests/test_emitter.py: single_head :1917, multi_block :1983, causal :2359 / :2369,
# causal_attention_gpu :5574, flash_attention_gpu :5647).
TEMPLATE_TOL = {"test_flash_attention_single_head": (1e-3, 1e-2), "test_flash_attention_multi_block": (1e-2, 5e-2),
                "test_flash_attention_causal": (1e-3, 2e-2), "test_causal_attention_gpu": (5e-2, 0.0),
                "test_flash_attention_gpu": (1e-1, 0.0)}


@pytest.mark.parametrize("name", sorted(TEMPLATE_TOL))
def test_template_golden(cuda, name):
    """The reference template tests' fp32 buffers (head_dim 64 runs the tf32
    tcgen05 kernel, head_dim 8 the CUDA-core kernel) at the reference's own
    tolerance."""
    import b200kern as bk
    g, rec = golden("ref_" + name), REF_TESTS[name]
    Q, K, V = (torch.tensor(g[n], device=cuda) for n in "qkv")
    out = bk.flash_attention_template(Q, K, V, rec["seq_len"], rec["scale"], rec["head_dim"], causal=rec["causal"])
    ref = (g["expected"] if "expected" in g else g["out"]).reshape(-1)
    atol, rtol = TEMPLATE_TOL[name]
    err = np.abs(out.reshape(-1).cpu().numpy() - ref)
    assert (err < np.maximum(atol, rtol * np.abs(ref))).all(), f"max err {err.max():.3g}"


@pytest.mark.parametrize("name", ["test_gqa_attention", "test_gqa_attention_gpu"])
def test_gqa_decode_golden(cuda, name):
    import b200kern as bk
    g, rec = golden("ref_" + name), REF_TESTS[name]
    out = bk.gqa_attention(torch.tensor(g["q"], device=cuda), torch.tensor(g["k"], device=cuda),
                           torch.tensor(g["v"], device=cuda), rec["seq_len"], rec["scale"], rec["n_q_per_kv"])
    ref = g["expected"] if "expected" in g else g["out"]
    assert np.abs(out.reshape(-1).cpu().numpy() - ref.reshape(-1)).max() < 1e-3


def _ref_torch(q, k, v, causal, scale=None):
    """fp32 reference on the GPU, per (b, h) to bound memory."""
    B, Hq, S, D = q.shape
    rep = Hq // k.shape[1]
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    out = torch.empty(B, Hq, S, D, device=q.device, dtype=torch.float32)
    for b in range(B):
        for h in range(Hq):
            s = (q[b, h].float() * scale) @ k[b, h // rep].float().t()
            if causal:
                s = s.masked_fill(torch.ones(S, k.shape[2], device=q.device, dtype=torch.bool).triu(1), float("-inf"))
            out[b, h] = torch.softmax(s, -1).nan_to_num(0.0) @ v[b, h // rep].float()
    return out


@pytest.mark.parametrize("D", [128, 64])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,Hq,Hkv,S,causal", [(1, 1, 1, 128, False), (1, 2, 2, 256, True), (2, 4, 2, 384, True),
                                               (1, 4, 1, 200, False), (1, 2, 1, 1000, True), (1, 8, 2, 2048, True)])
def test_fa_tcgen05(cuda, D, dtype, B, Hq, Hkv, S, causal):
    import b200kern as bk
    g = torch.Generator().manual_seed(S + Hq + D)
    q = (torch.randn(B, Hq, S, D, generator=g) * 0.5).to(dtype).to(cuda)
    k = (torch.randn(B, Hkv, S, D, generator=g) * 0.5).to(dtype).to(cuda)
    v = (torch.randn(B, Hkv, S, D, generator=g) * 0.5).to(dtype).to(cuda)
    out = bk.flash_attention(q, k, v, causal=causal)
    _close(out, _ref_torch(q, k, v, causal))


@pytest.mark.parametrize("B,Hq,Hkv,S,causal,window", [(1, 1, 1, 128, False, 0), (2, 8, 8, 1024, True, 0),
                                                      (1, 4, 2, 300, True, 0), (1, 4, 1, 777, False, 0),
                                                      (1, 2, 2, 640, True, 100), (1, 4, 2, 2048, True, 0)])
def test_fa_tf32_d64(cuda, B, Hq, Hkv, S, causal, window):
    """fp32 q / k / v with head dim 64 (the reference template's default) on
    the tcgen05 kernel with tf32 operands: fp32 output within rtol = atol =
    1e-2 of the float64 oracle (N(0,1) inputs, so logits of order 1)."""
    import b200kern as bk
    g = torch.Generator().manual_seed(S + Hq + window)
    q = torch.randn(B, Hq, S, 64, generator=g)
    k = torch.randn(B, Hkv, S, 64, generator=g)
    v = torch.randn(B, Hkv, S, 64, generator=g)
    out = bk.flash_attention(q.to(cuda), k.to(cuda), v.to(cuda), causal=causal, window=window)
    assert out.dtype == torch.float32
    ref = oatt.attention(q.double().numpy(), k.double().numpy(), v.double().numpy(), causal=causal, window=window)
    _close(out.cpu(), torch.from_numpy(ref))


def test_fa_tcgen05_strided_and_large_logits(cuda):
    """[B, S, H, D] storage viewed as [B, H, S, D]; large logits exercise the
    lazy O rescale (running max growing by > 2^8 across blocks)."""
    import b200kern as bk
    g = torch.Generator().manual_seed(3)
    base = torch.randn(2, 512, 4, 128, generator=g)
    base[:, 300:] *= 6.0
    q = base.bfloat16().to(cuda).transpose(1, 2)
    k = (torch.randn(2, 512, 4, 128, generator=g) * 2).bfloat16().to(cuda).transpose(1, 2)
    v = torch.randn(2, 512, 4, 128, generator=g).bfloat16().to(cuda).transpose(1, 2)
    for causal in (False, True):
        out = bk.flash_attention(q, k, v, causal=causal)
        _close(out, _ref_torch(q, k, v, causal))


def test_fa_oracle_small_bf16(cuda):
    """tcgen05 path vs the float64 numpy oracle on one small GQA case."""
    import b200kern as bk
    g = torch.Generator().manual_seed(11)
    q = (torch.randn(1, 4, 256, 128, generator=g) * 0.5).bfloat16()
    k = (torch.randn(1, 2, 256, 128, generator=g) * 0.5).bfloat16()
    v = (torch.randn(1, 2, 256, 128, generator=g) * 0.5).bfloat16()
    out = bk.flash_attention(q.to(cuda), k.to(cuda), v.to(cuda), causal=True).float().cpu()
    ref = oatt.attention(q.double().numpy(), k.double().numpy(), v.double().numpy(), causal=True)
    _close(out, torch.from_numpy(ref))


def test_fa_c0_config(cuda):
    """BASELINE configs[0] (the reference's CPU-runnable case): fp32
    [2, 8, 1024, 64], causal, scale 1/8, q then k then v ~ N(0, 1) from
    seed 0, against the float64 restatement of _ref_attention.  Runs the
    tcgen05 kernel with tf32 operands (10-bit mantissa, fp32 accumulate and
    softmax); north-star tolerance rtol = atol = 1e-2."""
    import b200kern as bk
    torch.manual_seed(0)
    q = torch.randn(2, 8, 1024, 64, dtype=torch.float32)
    k = torch.randn(2, 8, 1024, 64, dtype=torch.float32)
    v = torch.randn(2, 8, 1024, 64, dtype=torch.float32)
    o = bk.flash_attention(q.to(cuda), k.to(cuda), v.to(cuda), causal=True, scale=0.125)
    ref = oatt.attention(q.double().numpy(), k.double().numpy(), v.double().numpy(), causal=True, scale=0.125)
    np.testing.assert_allclose(o.double().cpu().numpy(), ref, rtol=1e-2, atol=1e-2)


def _ref_window(q, k, v, window):
    """fp32 causal sliding-window attention: key j visible to query i iff i - window < j <= i."""
    rep = q.shape[1] // k.shape[1]
    qf, kf, vf = q.float(), k.repeat_interleave(rep, 1).float(), v.repeat_interleave(rep, 1).float()
    s = qf @ kf.transpose(-1, -2) / math.sqrt(q.shape[-1])
    i = torch.arange(q.shape[2], device=q.device)[:, None]
    j = torch.arange(k.shape[2], device=q.device)[None, :]
    s = s.masked_fill((j > i) | (j <= i - window), float("-inf"))
    return torch.softmax(s, -1) @ vf


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,Hq,Hkv,S,window", [(1, 2, 2, 384, 1), (1, 2, 1, 384, 64), (2, 4, 2, 1000, 128),
                                               (1, 4, 2, 1000, 200), (1, 2, 2, 2048, 256), (1, 8, 2, 2048, 1000),
                                               (1, 2, 1, 512, 4096), (1, 2, 2, 700, 129)])
def test_fa_window_tcgen05(cuda, dtype, B, Hq, Hkv, S, window):
    """Sliding-window prefill on the tcgen05 kernel (D = 128): windows below,
    at, between and above the 128-key tile, and one wider than the sequence
    (= plain causal)."""
    import b200kern as bk
    g = torch.Generator().manual_seed(S + window)
    q = (torch.randn(B, Hq, S, 128, generator=g) * 0.5).to(dtype).to(cuda)
    k = (torch.randn(B, Hkv, S, 128, generator=g) * 0.5).to(dtype).to(cuda)
    v = (torch.randn(B, Hkv, S, 128, generator=g) * 0.5).to(dtype).to(cuda)
    out = bk.flash_attention(q, k, v, causal=True, window=window)
    _close(out, _ref_window(q, k, v, window))


def test_fa_window_large_logits(cuda):
    """Window plus the lazy O rescale: a running max that grows by > 2^8
    inside the window."""
    import b200kern as bk
    g = torch.Generator().manual_seed(5)
    base = torch.randn(1, 4, 768, 128, generator=g)
    base[:, :, 400:] *= 6.0
    q = base.bfloat16().to(cuda)
    k = (torch.randn(1, 4, 768, 128, generator=g) * 2).bfloat16().to(cuda)
    v = torch.randn(1, 4, 768, 128, generator=g).bfloat16().to(cuda)
    out = bk.flash_attention(q, k, v, causal=True, window=300)
    _close(out, _ref_window(q, k, v, 300))


@pytest.mark.parametrize("D,dtype", [(64, torch.float32), (96, torch.bfloat16), (128, torch.float32)])
def test_fa_window_generic_vs_oracle(cuda, D, dtype):
    """The CUDA-core kernel (D != 128 or fp32) with a window vs the float64 oracle."""
    import b200kern as bk
    g = torch.Generator().manual_seed(D)
    q = torch.randn(1, 4, 300, D, generator=g).to(dtype)
    k = torch.randn(1, 2, 300, D, generator=g).to(dtype)
    v = torch.randn(1, 2, 300, D, generator=g).to(dtype)
    out = bk.flash_attention(q.to(cuda), k.to(cuda), v.to(cuda), causal=True, window=37).double().cpu()
    ref = oatt.attention(q.double().numpy(), k.double().numpy(), v.double().numpy(), causal=True, window=37)
    _close(out, torch.from_numpy(ref))


def test_fa_window_tcgen05_vs_oracle(cuda):
    """tcgen05 window path vs the float64 oracle."""
    import b200kern as bk
    g = torch.Generator().manual_seed(13)
    q = (torch.randn(1, 4, 640, 128, generator=g) * 0.5).bfloat16()
    k = (torch.randn(1, 2, 640, 128, generator=g) * 0.5).bfloat16()
    v = (torch.randn(1, 2, 640, 128, generator=g) * 0.5).bfloat16()
    out = bk.flash_attention(q.to(cuda), k.to(cuda), v.to(cuda), causal=True, window=160).float().cpu()
    ref = oatt.attention(q.double().numpy(), k.double().numpy(), v.double().numpy(), causal=True, window=160)
    _close(out, torch.from_numpy(ref))


def test_fa_no_bounded_wait_ran_out(cuda):
    import ctypes
    from b200kern import _lib
    code = ctypes.c_uint(0)
    st = _lib.load().b2_device_error(torch.cuda.current_stream().cuda_stream, ctypes.byref(code))
    assert st == 0 and code.value == 0, hex(code.value)

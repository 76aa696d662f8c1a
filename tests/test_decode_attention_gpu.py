"""Parity of the split-KV decode attention kernel (contiguous and paged KV
caches) with the oracle.  Reference golden cases use the reference tests'
own tolerances or tighter (1e-3 abs on their fp32 data); the rest use the
north-star element-wise rtol = atol = 1e-2 against float64."""
import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden
from oracle import attention as oatt

pytestmark = pytest.mark.gpu
MANIFEST = json.load(open(os.path.join(GOLDEN, "manifest.json")))
REF = {r["test"]: r for r in MANIFEST["reference_tests"]}


def _ref(g, name):
    return g["expected"] if "expected" in g else g["out"]


@pytest.mark.parametrize("name", ["test_kv_cache_attention", "test_kv_cache_attention_gpu"])
def test_kv_cache_golden(cuda, name):
    import b200kern as bk
    g, rec = golden("ref_" + name), REF[name]
    t = lambda a: torch.tensor(a, device=cuda)
    out = bk.kv_cache_attention(t(g["q"]), t(g["k"]), t(g["v"]), rec["seq_len"], rec["scale"])
    assert np.abs(out.reshape(-1).cpu().numpy() - _ref(g, name).reshape(-1)).max() < 1e-3


def test_batched_decode_golden(cuda):
    import b200kern as bk
    name = "test_batched_kv_decode"
    g, rec = golden("ref_" + name), REF[name]
    t = lambda a: torch.tensor(a, device=cuda)
    out = bk.batched_kv_decode(t(g["q"]), t(g["k"]), t(g["v"]), t(g["seq_lens"]), rec["max_seq_len"])
    assert np.abs(out.reshape(-1).cpu().numpy() - _ref(g, name).reshape(-1)).max() < 1e-3


@pytest.mark.parametrize("name", ["test_paged_attention", "test_paged_attention_partial_page",
                                  "test_paged_attention_gpu", "test_multi_head_paged_attention"])
def test_paged_golden(cuda, name):
    import b200kern as bk
    g, rec = golden("ref_" + name), REF[name]
    t = lambda a: torch.tensor(a, device=cuda)
    out = bk.paged_attention(t(g["q"]), t(g["k"]), t(g["v"]), t(g["page_table"]), rec["seq_len"], rec["n_pages"],
                             rec["page_size"])
    assert np.abs(out.reshape(-1).cpu().numpy() - _ref(g, name).reshape(-1)).max() < 1e-3


def test_fp16_kv_golden(cuda):
    import b200kern as bk
    name = "test_fp16_kv_attention"
    g, rec = golden("ref_" + name), REF[name]
    q = torch.tensor(g["q"], device=cuda)  # fp32 query
    k = torch.tensor(g["k"], device=cuda).half()  # the reference stores the cache in fp16
    v = torch.tensor(g["v"], device=cuda).half()
    out = bk.kv_cache_attention(q, k, v, rec["seq_len"], rec["scale"])
    assert out.dtype == torch.float32
    assert np.abs(out.reshape(-1).cpu().numpy() - _ref(g, name).reshape(-1)).max() < 1e-3


def _close(out, ref, tol=1e-2):
    err = np.abs(out - ref)
    assert (err <= tol + tol * np.abs(ref)).all(), f"max err {err.max():.4g}"


@pytest.mark.parametrize("qdt,kvdt", [(torch.bfloat16, torch.bfloat16), (torch.float16, torch.float16),
                                      (torch.float32, torch.float16), (torch.float32, torch.float32)])
@pytest.mark.parametrize("B,Hq,Hkv,S,D", [(1, 8, 8, 100, 64), (3, 32, 8, 4096, 128), (2, 16, 1, 777, 128),
                                          (64, 8, 2, 300, 256), (40, 16, 4, 1000, 128)])
def test_decode_contiguous(cuda, qdt, kvdt, B, Hq, Hkv, S, D):
    import b200kern as bk
    g = torch.Generator().manual_seed(B * 1000 + S)
    q = torch.randn(B, Hq, D, generator=g).to(qdt)
    k = torch.randn(B, Hkv, S, D, generator=g).to(kvdt)
    v = torch.randn(B, Hkv, S, D, generator=g).to(kvdt)
    lens = torch.randint(0, S + 1, (B,), generator=g, dtype=torch.int32)
    lens[0] = S
    out = bk.decode_attention(q.to(cuda), k.to(cuda), v.to(cuda), lens.to(cuda))
    ref = oatt.decode(q.double().numpy(), k.double().numpy(), v.double().numpy(), lens.numpy())
    _close(out.double().cpu().numpy(), ref)


def test_decode_paged_random_tables(cuda):
    """Paged pool shared by the batch, shuffled page tables, ragged lengths."""
    import b200kern as bk
    g = torch.Generator().manual_seed(5)
    B, Hq, Hkv, D, ps, max_pages = 4, 16, 4, 128, 16, 40
    n_phys = B * max_pages
    kp = torch.randn(n_phys, ps, Hkv, D, generator=g).bfloat16()
    vp = torch.randn(n_phys, ps, Hkv, D, generator=g).bfloat16()
    table = torch.randperm(n_phys, generator=g).reshape(B, max_pages).to(torch.int32)
    lens = torch.tensor([640, 1, 333, 0], dtype=torch.int32)
    q = torch.randn(B, Hq, D, generator=g).bfloat16()
    out = bk.decode_attention(q.to(cuda), kp.to(cuda), vp.to(cuda), lens.to(cuda), page_table=table.to(cuda))
    kc = np.zeros((B, Hkv, max_pages * ps, D))
    vc = np.zeros_like(kc)
    for b in range(B):
        n = int(lens[b])
        kc[b, :, :n] = oatt.gather_pages(kp.double().numpy(), table[b].numpy(), n).transpose(1, 0, 2)
        vc[b, :, :n] = oatt.gather_pages(vp.double().numpy(), table[b].numpy(), n).transpose(1, 0, 2)
    ref = oatt.decode(q.double().numpy(), kc, vc, lens.numpy())
    _close(out.double().cpu().numpy(), ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_decode_paged_full_and_overlong(cuda, dtype):
    """Sequences that fill every page of their table row exactly, and one whose
    seq_len claims more keys than its pages hold: that one is clamped to the
    table's capacity (max_pages * page_size keys), never read past its row."""
    import b200kern as bk
    g = torch.Generator().manual_seed(21)
    B, Hq, Hkv, D, ps, max_pages = 3, 8, 2, 128, 16, 6
    cap = ps * max_pages
    n_phys = B * max_pages + 2
    kp = torch.randn(n_phys, ps, Hkv, D, generator=g).to(dtype)
    vp = torch.randn(n_phys, ps, Hkv, D, generator=g).to(dtype)
    table = torch.randperm(n_phys, generator=g)[:B * max_pages].reshape(B, max_pages).to(torch.int32)
    lens = torch.tensor([cap, cap, cap + 50], dtype=torch.int32)
    q = torch.randn(B, Hq, D, generator=g).to(dtype)
    out = bk.decode_attention(q.to(cuda), kp.to(cuda), vp.to(cuda), lens.to(cuda), page_table=table.to(cuda))
    kc = np.zeros((B, Hkv, cap, D))
    vc = np.zeros_like(kc)
    for b in range(B):
        kc[b] = oatt.gather_pages(kp.double().numpy(), table[b].numpy(), cap).transpose(1, 0, 2)
        vc[b] = oatt.gather_pages(vp.double().numpy(), table[b].numpy(), cap).transpose(1, 0, 2)
    ref = oatt.decode(q.double().numpy(), kc, vc, np.minimum(lens.numpy(), cap))
    _close(out.double().cpu().numpy(), ref)


def test_gqa_decode_matches_flash_attention(cuda):
    """Decode of the last position == the last row of causal prefill attention."""
    import b200kern as bk
    g = torch.Generator().manual_seed(8)
    q = (torch.randn(2, 8, 512, 128, generator=g) * 0.5).bfloat16().to(cuda)
    k = (torch.randn(2, 2, 512, 128, generator=g) * 0.5).bfloat16().to(cuda)
    v = (torch.randn(2, 2, 512, 128, generator=g) * 0.5).bfloat16().to(cuda)
    full = bk.flash_attention(q, k, v, causal=True)[:, :, -1]
    dec = bk.decode_attention(q[:, :, -1].contiguous(), k, v, 512)
    _close(dec.double().cpu().numpy(), full.double().cpu().numpy(), tol=2e-2)


# ---------------------------------------------------------------------------
# sliding window, fused RoPE, repeat_kv
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("name", ["test_sliding_window_attention", "test_sliding_window_attention_gpu"])
def test_sliding_window_golden(cuda, name):
    import b200kern as bk
    g, rec = golden("ref_" + name), REF[name]
    t = lambda a: torch.tensor(a, device=cuda)
    out = bk.sliding_window_attention(t(g["q"]), t(g["k"]), t(g["v"]), rec["q_pos"], rec["seq_len"], rec["window"])
    ref = g["expected"] if "expected" in g else g["out"]
    assert np.abs(out.reshape(-1).cpu().numpy() - ref.reshape(-1)).max() < 1e-3


def test_rope_golden(cuda):
    import b200kern as bk
    g, rec = golden("ref_test_rope_attention"), REF["test_rope_attention"]
    t = lambda a: torch.tensor(a, device=cuda)
    out = bk.rope_attention(t(g["q"]), t(g["k"]), t(g["v"]), t(g["freqs"]), rec["seq_len"], rec["q_pos"])
    assert np.abs(out.reshape(-1).cpu().numpy() - g["out"].reshape(-1)).max() < 1e-4


def test_repeat_kv_golden(cuda):
    import b200kern as bk
    g = golden("ref_test_repeat_kv")
    out = bk.repeat_kv(torch.tensor(g["x"], device=cuda), REF["test_repeat_kv"]["n_rep"])
    assert np.array_equal(out.reshape(-1).cpu().numpy(), g["out"].reshape(-1))  # a copy: bit-exact


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("paged", [False, True])
def test_decode_window_rope_large(cuda, dt, paged):
    """Sliding window + RoPE together, ragged lengths and query positions,
    GQA, contiguous and paged caches, tensor-core (16-bit) and generic (fp32)."""
    import b200kern as bk
    g = torch.Generator().manual_seed(11 + paged)
    B, Hq, Hkv, D, S, W = 3, 16, 4, 128, 2500, 700
    q = torch.randn(B, Hq, D, generator=g).to(dt)
    k = torch.randn(B, Hkv, S, D, generator=g).to(dt)
    v = torch.randn(B, Hkv, S, D, generator=g).to(dt)
    lens = torch.tensor([2500, 1999, 300], dtype=torch.int32)
    qpos = torch.tensor([2499, 1200, 299], dtype=torch.int32)
    freqs = 1.0 / 10000.0 ** (torch.arange(0, D, 2, dtype=torch.float64) / D)
    if paged:
        ps = 16
        npg = S // ps + 1
        perm = torch.randperm(B * npg, generator=g).to(torch.int32).reshape(B, npg)
        kp = torch.zeros(B * npg, ps, Hkv, D, dtype=dt)
        vp = torch.zeros(B * npg, ps, Hkv, D, dtype=dt)
        for b in range(B):
            for pg in range(npg):
                lo, hi = pg * ps, min(S, pg * ps + ps)
                if lo >= hi:
                    continue
                kp[perm[b, pg], : hi - lo] = k[b, :, lo:hi].transpose(0, 1)
                vp[perm[b, pg], : hi - lo] = v[b, :, lo:hi].transpose(0, 1)
        out = bk.decode_attention(q.to(cuda), kp.to(cuda), vp.to(cuda), lens.to(cuda), page_table=perm.to(cuda),
                                  q_pos=qpos, window=W, rope_freqs=freqs.float())
    else:
        out = bk.decode_attention(q.to(cuda), k.to(cuda), v.to(cuda), lens.to(cuda), q_pos=qpos, window=W,
                                  rope_freqs=freqs.float())
    ref = oatt.decode(q.double().numpy(), k.double().numpy(), v.double().numpy(), lens.numpy(),
                      q_pos=qpos.numpy(), window=W, rope_freqs=freqs.float().double().numpy())
    _close(out.double().cpu().numpy(), ref, tol=2e-2 if dt != torch.float32 else 1e-2)


@pytest.mark.parametrize("W", [1, 64, 5000])
def test_decode_window_edges(cuda, W):
    """Window of one key, a window inside one tile, a window wider than the cache."""
    import b200kern as bk
    g = torch.Generator().manual_seed(W)
    B, Hq, Hkv, D, S = 2, 8, 8, 64, 1000
    q = torch.randn(B, Hq, D, generator=g).bfloat16()
    k = torch.randn(B, Hkv, S, D, generator=g).bfloat16()
    v = torch.randn(B, Hkv, S, D, generator=g).bfloat16()
    lens = torch.tensor([1000, 517], dtype=torch.int32)
    out = bk.decode_attention(q.to(cuda), k.to(cuda), v.to(cuda), lens.to(cuda), window=W)
    ref = oatt.decode(q.double().numpy(), k.double().numpy(), v.double().numpy(), lens.numpy(), window=W)
    _close(out.double().cpu().numpy(), ref)


@pytest.mark.parametrize("dt,shape,rep", [(torch.bfloat16, (8, 4096, 128), 4), (torch.float32, (2, 5, 3), 3),
                                          (torch.float16, (2, 3, 8, 100, 64), 2)])
def test_repeat_kv_shapes(cuda, dt, shape, rep):
    import b200kern as bk
    x = torch.randn(*shape).to(dt).to(cuda)
    out = bk.repeat_kv(x, rep)
    assert torch.equal(out, x.repeat_interleave(rep, dim=-3))


def test_decode_no_bounded_wait_ran_out(cuda):
    import ctypes
    from b200kern import _lib
    code = ctypes.c_uint(0)
    st = _lib.load().b2_device_error(torch.cuda.current_stream().cuda_stream, ctypes.byref(code))
    assert st == 0 and code.value == 0, hex(code.value)

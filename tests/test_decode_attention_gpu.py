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

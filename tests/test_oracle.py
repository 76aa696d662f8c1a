"""Pin the CPU oracle against the reference's golden vectors (no GPU).

The fixtures in tests/golden/ were produced by tests/golden/make_golden.py:
the reference's own hot-path tests were executed against this oracle (and
passed their own assertions), and the reference's torch _ref_attention
(tests/test_flash_attention.py:107-118) was run on its seeded shapes.
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, golden
from oracle import attention as oatt
from oracle import quant as oq

MANIFEST = json.load(open(os.path.join(GOLDEN, "manifest.json")))
REF_TESTS = {r["test"]: r for r in MANIFEST["reference_tests"]}


def test_every_reference_test_accepted_the_oracle():
    assert len(REF_TESTS) == 23
    for name, rec in REF_TESTS.items():
        assert rec["reference_test_passed"], (name, rec["error"])


@pytest.mark.parametrize("name", [n for n, r in REF_TESTS.items() if r["has_expected"]])
def test_oracle_matches_reference_expected(name):
    """The reference test's own `expected` list (pure-Python float64 loop over
    unrounded inputs) vs the oracle on the float32 buffers it bound."""
    g = golden("ref_" + name)
    rec = REF_TESTS[name]
    if rec["kernel"] == "int4_matmul":
        out = oq.int4_matmul_ref_layout(g["x"], g["w"], g["s"], g["z"], rec["group_size"])
    elif rec["kernel"] == "int8_matmul":
        out = oq.int8_matmul(g["x"], g["w"], g["s"], g["z"])
    elif rec["kernel"] in ("flash_attention", "causal_attention"):
        out = oatt.flash_attention_template(g["q"], g["k"], g["v"], rec["seq_len"], rec["scale"],
                                            rec["head_dim"], causal=rec["causal"])
    elif rec["kernel"] == "gqa_attention":
        out = oatt.gqa_decode(g["q"], g["k"], g["v"], rec["seq_len"], rec["scale"], rec["n_q_per_kv"])
    elif rec["kernel"] in ("kv_cache_attention", "fp16_kv_attention"):
        out = oatt.decode(g["q"][None], g["k"][None], g["v"][None], [rec["seq_len"]], rec["scale"])
    elif rec["kernel"] == "sliding_window_attention":
        out = oatt.sliding_window_decode(g["q"], g["k"], g["v"], rec["q_pos"], rec["seq_len"], rec["window"])
    elif rec["kernel"] == "rope_attention":
        out = oatt.rope_decode(g["q"], g["k"], g["v"], g["freqs"], rec["seq_len"], rec["q_pos"])
    elif rec["kernel"] == "repeat_kv":
        out = oatt.repeat_kv(g["x"], rec["n_rep"])
    elif rec["kernel"] == "batched_kv_decode":
        out = oatt.decode(g["q"], g["k"], g["v"], g["seq_lens"], 1.0 / np.sqrt(rec["head_dim"]))
    else:  # paged
        kc = oatt.gather_pages(g["k"], g["page_table"], rec["seq_len"]).transpose(1, 0, 2)
        vc = oatt.gather_pages(g["v"], g["page_table"], rec["seq_len"]).transpose(1, 0, 2)
        out = oatt.decode(g["q"][None], kc[None], vc[None], [rec["seq_len"]], 1.0 / np.sqrt(rec["head_dim"]))
    np.testing.assert_allclose(out.reshape(-1), g["expected"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", ["test_sliding_window_attention", "test_rope_attention", "test_repeat_kv"])
def test_oracle_reproduces_saved_outputs(name):
    """Reference tests that check inline (no `expected` list): the saved
    output is what the reference test accepted; the oracle must reproduce it."""
    g, rec = golden("ref_" + name), REF_TESTS[name]
    if name == "test_repeat_kv":
        out = oatt.repeat_kv(g["x"], rec["n_rep"])
    elif name == "test_rope_attention":
        out = oatt.rope_decode(g["q"], g["k"], g["v"], g["freqs"], rec["seq_len"], rec["q_pos"])
    else:
        out = oatt.sliding_window_decode(g["q"], g["k"], g["v"], rec["q_pos"], rec["seq_len"], rec["window"])
    np.testing.assert_allclose(out.reshape(-1), g["out"], rtol=1e-6, atol=1e-6)


def test_rope_rotation_is_a_rotation():
    """RoPE preserves pair norms and composes additively in position."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((5, 64))
    f = 1.0 / 10000.0 ** (2.0 * np.arange(32) / 64)
    r = oatt.rope_rotate(x, 7, f)
    np.testing.assert_allclose((r[:, 0::2] ** 2 + r[:, 1::2] ** 2), (x[:, 0::2] ** 2 + x[:, 1::2] ** 2), atol=1e-12)
    np.testing.assert_allclose(oatt.rope_rotate(oatt.rope_rotate(x, 3, f), 4, f), r, atol=1e-12)


@pytest.mark.parametrize("rec", MANIFEST["triton_fa"], ids=lambda r: r["name"])
def test_oracle_matches_ref_attention(rec):
    g = golden(rec["name"])
    out = oatt.attention(g["q"], g["k"], g["v"], causal=rec["causal"])
    np.testing.assert_allclose(out, g["out"], rtol=1e-5, atol=1e-5)


def test_int4_ref_layout_nibble_order():
    """Even k in the low nibble, odd k in the high (_msl_templates.py:2725-2732)."""
    packed = np.array([[0x21, 0x43]], dtype=np.uint8)
    assert oq.unpack_int4_ref(packed).tolist() == [[1, 2, 3, 4]]


def test_gptq_roundtrip_and_repack_bit_exact():
    rng = np.random.default_rng(0)
    q = rng.integers(0, 16, size=(64, 24))  # [K, N]
    words = oq.pack_int4_gptq(q)
    assert words.dtype == np.int32 and words.shape == (8, 24)
    assert np.array_equal(oq.unpack_int4_gptq(words), q)
    ref = oq.pack_int4_ref(q.T)
    assert np.array_equal(oq.unpack_int4_ref(ref), q.T)
    assert np.array_equal(oq.ref_to_gptq(ref), words)


def test_dequant_exact_in_fp32():
    """(q - 8) * s with fp16 scales is exact in fp32: compare with float64."""
    rng = np.random.default_rng(1)
    q = rng.integers(0, 16, size=(256, 16))
    s = (np.abs(rng.standard_normal((2, 16))) * 0.02 + 1e-3).astype(np.float16)
    w32 = oq.dequant_int4(q, s, None, 128, dtype=np.float32)
    w64 = oq.dequant_int4(q, s.astype(np.float64), None, 128, dtype=np.float64)
    assert np.array_equal(w32.astype(np.float64), w64)


def test_asymmetric_zero_matches_loop():
    """Vectorised oracle vs a direct per-element loop (test_emitter.py:6170-6185)."""
    rng = np.random.default_rng(2)
    M, N, K, G = 2, 4, 16, 8
    x = rng.standard_normal((M, K))
    q = rng.integers(0, 16, size=(N, K))
    s = rng.uniform(0.1, 0.5, size=(N, K // G))
    z = rng.uniform(0, 8, size=(N, K // G))
    exp = np.zeros((M, N))
    for i in range(M):
        for j in range(N):
            exp[i, j] = sum(x[i, k] * (q[j, k] - z[j, k // G]) * s[j, k // G] for k in range(K))
    out = oq.int4_matmul_ref_layout(x, oq.pack_int4_ref(q), s, z, G)
    np.testing.assert_allclose(out, exp, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("rec", MANIFEST["kda"], ids=lambda r: r["name"])
def test_kda_oracle_matches_fla(rec):
    """KDA oracle vs flash-linear-attention 0.5.1's naive recurrence (the
    reference has no KDA; fla is the operator's defining library)."""
    from oracle import kda as okda
    g = golden(rec["name"])
    o, S = okda.recurrent(g["q"], g["k"], g["v"], g["g"], g["beta"], initial_state=g.get("s0"))
    np.testing.assert_allclose(o, g["o"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(S, g["S"], rtol=1e-4, atol=1e-4)


def test_oracle_attention_window_matches_loop():
    """The vectorised window mask vs a per-query loop over keys
    max(0, i + 1 - window) .. i (the decode window's start rule)."""
    r = np.random.default_rng(7)
    q, k, v = (r.standard_normal((1, 2, 40, 8)) for _ in range(3))
    w = 6
    got = oatt.attention(q, k, v, causal=True, window=w)
    s = q @ np.swapaxes(k, -1, -2) / np.sqrt(8)
    want = np.zeros_like(q)
    for i in range(40):
        js = np.arange(max(0, i + 1 - w), i + 1)
        p = np.exp(s[..., i, js] - s[..., i, js].max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True)
        want[..., i, :] = np.einsum("bhj,bhjd->bhd", p, v[:, :, js, :])
    np.testing.assert_allclose(got, want, rtol=1e-12, atol=1e-12)
    np.testing.assert_array_equal(oatt.attention(q, k, v, causal=True, window=40),
                                  oatt.attention(q, k, v, causal=True))

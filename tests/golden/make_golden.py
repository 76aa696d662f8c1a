"""Generate the golden fixtures in this folder from the reference itself.

Run in a container that has the reference checkout (read-only); its path
must be given in the REFERENCE_ROOT environment variable.  The GPU box never
runs this.

Two sources of golden vectors:
 1. The reference's own hot-path tests in tests/test_emitter.py are executed
    unmodified, with a stand-in for their Metal runner: the reference
    MetalKernelRunner's buffer packing/reading is reused as-is, but the
    compile/dispatch steps evaluate the CPU oracle (oracle/quant.py,
    oracle/attention.py) on the bound buffers.  Each reference test then
    checks the oracle's output against its own pure-Python reference loop
    and tolerance.  The buffers (inputs) and outputs of every dispatch are
    saved, plus the test's own `expected` list when it builds one.
 2. The reference's torch oracle _ref_attention
    (tests/test_flash_attention.py:107-118) on the seeded shapes of
    TestFlashAttention (torch.manual_seed(42), fp32 randn).

Usage: python tests/golden/make_golden.py
"""
import json
import math
import os
import re
import sys
import types

import numpy as np

sys.dont_write_bytecode = True
HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("REFERENCE_ROOT")
if not REF:
    raise SystemExit("set REFERENCE_ROOT to the reference checkout (bledden/triton-metal)")
sys.path.insert(0, REPO)
from oracle import attention as oatt  # noqa: E402
from oracle import quant as oq  # noqa: E402


# --------------------------------------------------------------------------
# stand-in Metal runtime (host memory buffers; dispatch = CPU oracle)
# --------------------------------------------------------------------------
class _Contents:
    def __init__(self, mem):
        self._mem = mem

    def as_buffer(self, n):
        return memoryview(self._mem)[:n]


class FakeBuffer:
    def __init__(self, n):
        self.mem = bytearray(n)

    def contents(self):
        return _Contents(self.mem)

    def f32(self):
        return np.frombuffer(bytes(self.mem), dtype=np.float32)

    def u32(self):
        return int(np.frombuffer(bytes(self.mem[:4]), dtype=np.uint32)[0])


class FakeDevice:
    def newBufferWithLength_options_(self, n, opts):
        return FakeBuffer(n)


DISPATCHES = []


class Pipeline:
    def __init__(self, name, msl):
        self.name, self.msl = name, msl


def _const(msl, pattern):
    m = re.search(pattern, msl)
    return int(m.group(1)) if m else None


def execute(pipe, bufs):
    name, msl = pipe.name, pipe.msl
    rec = {"kernel": name}
    if name in ("int4_matmul", "int8_matmul"):
        x_b, w_b, o_b, s_b, z_b, m_b, n_b, k_b = bufs
        M, N, K = m_b.u32(), n_b.u32(), k_b.u32()
        x = x_b.f32()[: M * K].reshape(M, K)
        if name == "int4_matmul":
            G = _const(msl, r"GROUP_SIZE = (\d+)u")
            ng = (K + G - 1) // G
            w = np.frombuffer(bytes(w_b.mem), dtype=np.uint8)[: N * K // 2].reshape(N, K // 2)
            s = s_b.f32()[: N * ng].reshape(N, ng)
            z = z_b.f32()[: N * ng].reshape(N, ng)
            out = oq.int4_matmul_ref_layout(x, w, s, z, G)
            rec.update(group_size=G)
        else:
            w = np.frombuffer(bytes(w_b.mem), dtype=np.int8)[: N * K].reshape(N, K)
            s = s_b.f32()[:N]
            z = z_b.f32()[:N]
            out = oq.int8_matmul(x, w, s, z)
        rec.update(M=M, N=N, K=K, x=x, w=w, s=s, z=z)
        ob = out.astype(np.float32).reshape(-1)
    elif name == "flash_attention":
        q_b, k_b, v_b, o_b, sl_b, sc_b = bufs
        S = sl_b.u32()
        scale = float(np.frombuffer(bytes(sc_b.mem[:4]), dtype=np.float32)[0])
        D = _const(msl, r"const uint D = (\d+)u")
        causal = "kv_pos_check" in msl
        n = len(q_b.mem) // 4
        q, k, v = q_b.f32(), k_b.f32(), v_b.f32()
        out = oatt.flash_attention_template(q, k, v, S, scale, D, causal=causal)
        rec.update(seq_len=S, scale=scale, head_dim=D, causal=causal, q=q, k=k, v=v)
        ob = out.astype(np.float32).reshape(-1)[:n]
    elif name == "causal_attention":
        q_b, k_b, v_b, o_b, sl_b = bufs
        S = sl_b.u32()
        D = _const(msl, r"query_pos \* (\d+)u")
        q, k, v = q_b.f32(), k_b.f32(), v_b.f32()
        out = oatt.flash_attention_template(q, k, v, S, 1.0 / math.sqrt(D), D, causal=True)
        rec.update(seq_len=S, scale=1.0 / math.sqrt(D), head_dim=D, causal=True, q=q, k=k, v=v)
        ob = out.astype(np.float32).reshape(-1)
    elif name == "gqa_attention":
        q_b, k_b, v_b, o_b, sl_b, sc_b = bufs
        S = sl_b.u32()
        scale = float(np.frombuffer(bytes(sc_b.mem[:4]), dtype=np.float32)[0])
        D = _const(msl, r"const uint D = (\d+)u")
        rep = _const(msl, r"const uint N_Q_PER_KV = (\d+)u")
        q = q_b.f32().reshape(-1, D)
        k, v = k_b.f32(), v_b.f32()
        out = oatt.gqa_decode(q, k, v, S, scale, rep)
        rec.update(seq_len=S, scale=scale, head_dim=D, n_q_per_kv=rep, q=q, k=k, v=v)
        ob = out.astype(np.float32).reshape(-1)
    elif name in ("kv_cache_attention", "fp16_kv_attention"):
        D = _const(msl, r"const uint D = (\d+)u")
        if name == "kv_cache_attention":
            q_b, k_b, v_b, o_b, sl_b, sc_b = bufs
            scale = float(np.frombuffer(bytes(sc_b.mem[:4]), dtype=np.float32)[0])
            k, v = k_b.f32(), v_b.f32()
        else:
            q_b, k_b, v_b, o_b, sl_b = bufs
            scale = 1.0 / math.sqrt(D)
            k = np.frombuffer(bytes(k_b.mem), dtype=np.float16).astype(np.float32)
            v = np.frombuffer(bytes(v_b.mem), dtype=np.float16).astype(np.float32)
        S = sl_b.u32()
        q = q_b.f32().reshape(-1, D)
        H = q.shape[0]
        k = k.reshape(H, -1, D)
        v = v.reshape(H, -1, D)
        out = oatt.decode(q[None], k[None], v[None], [S], scale)[0]
        rec.update(seq_len=S, scale=scale, head_dim=D, q=q, k=k, v=v)
        ob = out.astype(np.float32).reshape(-1)
    elif name == "batched_kv_decode":
        q_b, k_b, v_b, o_b, sl_b, ms_b, bs_b = bufs
        D = _const(msl, r"const uint D = (\d+)u")
        H = _const(msl, r"const uint N_HEADS = (\d+)u")
        Bsz, S = bs_b.u32(), ms_b.u32()
        lens = np.frombuffer(bytes(sl_b.mem), dtype=np.uint32)[:Bsz]
        q = q_b.f32()[: Bsz * H * D].reshape(Bsz, H, D)
        k = k_b.f32()[: Bsz * H * S * D].reshape(Bsz, H, S, D)
        v = v_b.f32()[: Bsz * H * S * D].reshape(Bsz, H, S, D)
        out = oatt.decode(q, k, v, lens, 1.0 / math.sqrt(D))
        rec.update(seq_lens=lens.astype(np.int64), max_seq_len=S, head_dim=D, q=q, k=k, v=v)
        ob = out.astype(np.float32).reshape(-1)
    elif name in ("paged_attention", "multi_head_paged_attention"):
        q_b, k_b, v_b, pt_b, o_b, sl_b, np_b = bufs
        D = _const(msl, r"const uint D = (\d+)u")
        ps = _const(msl, r"const uint PAGE_SIZE = (\d+)u")
        S, npg = sl_b.u32(), np_b.u32()
        table = np.frombuffer(bytes(pt_b.mem), dtype=np.uint32)[:npg]
        q = q_b.f32().reshape(-1, D)
        H = q.shape[0]
        kp = k_b.f32().reshape(-1, ps, H, D) if name.startswith("multi") else k_b.f32().reshape(-1, ps, 1, D)
        vp = v_b.f32().reshape(-1, ps, H, D) if name.startswith("multi") else v_b.f32().reshape(-1, ps, 1, D)
        kc = oatt.gather_pages(kp, table, S).transpose(1, 0, 2)  # [H, S, D]
        vc = oatt.gather_pages(vp, table, S).transpose(1, 0, 2)
        out = oatt.decode(q[None], kc[None], vc[None], [S], 1.0 / math.sqrt(D))[0]
        rec.update(seq_len=S, n_pages=npg, page_size=ps, head_dim=D, page_table=table.astype(np.int64),
                   q=q, k=kp, v=vp)
        ob = out.astype(np.float32).reshape(-1)
    elif name == "sliding_window_attention":
        q_b, k_b, v_b, o_b, qp_b, sl_b = bufs
        D = _const(msl, r"const uint D = (\d+)u")
        W = _const(msl, r"const uint WINDOW = (\d+)u")
        qp, S = qp_b.u32(), sl_b.u32()
        q, k, v = q_b.f32()[:D], k_b.f32()[: S * D], v_b.f32()[: S * D]
        out = oatt.sliding_window_decode(q, k, v, qp, S, W)
        rec.update(seq_len=S, q_pos=qp, window=W, head_dim=D, q=q, k=k.reshape(S, D), v=v.reshape(S, D))
        ob = out.astype(np.float32).reshape(-1)
    elif name == "rope_attention":
        q_b, k_b, v_b, f_b, o_b, sl_b, qp_b = bufs
        D = _const(msl, r"const uint D = (\d+)u")
        S, qp = sl_b.u32(), qp_b.u32()
        q, k, v = q_b.f32()[:D], k_b.f32()[: S * D], v_b.f32()[: S * D]
        freqs = f_b.f32()[: D // 2]
        out = oatt.rope_decode(q, k, v, freqs, S, qp)
        rec.update(seq_len=S, q_pos=qp, head_dim=D, q=q, k=k.reshape(S, D), v=v.reshape(S, D), freqs=freqs)
        ob = out.astype(np.float32).reshape(-1)
    elif name == "repeat_kv":
        i_b, o_b, h_b, sl_b, hd_b, nr_b = bufs
        H, S, D, R = h_b.u32(), sl_b.u32(), hd_b.u32(), nr_b.u32()
        x = i_b.f32()[: H * S * D].reshape(H, S, D)
        out = oatt.repeat_kv(x, R)
        rec.update(n_kv_heads=H, seq_len=S, head_dim=D, n_rep=R, x=x)
        ob = out.astype(np.float32).reshape(-1)
    else:
        raise KeyError(name)
    o_b.mem[: ob.nbytes] = ob.tobytes()
    rec["out"] = ob
    DISPATCHES.append(rec)


class FakeEncoder:
    def __init__(self):
        self.bufs = {}
        self.pipe = None

    def setComputePipelineState_(self, p):
        self.pipe = p

    def setBuffer_offset_atIndex_(self, buf, off, i):
        self.bufs[i] = buf

    def dispatchThreadgroups_threadsPerThreadgroup_(self, a, b):
        execute(self.pipe, [self.bufs[i] for i in sorted(self.bufs)])

    def endEncoding(self):
        pass


class FakeCmd:
    def computeCommandEncoder(self):
        return FakeEncoder()

    def commit(self):
        pass

    def waitUntilCompleted(self):
        pass

    def status(self):
        return 4  # MTLCommandBufferStatusCompleted


class FakeQueue:
    def commandBuffer(self):
        return FakeCmd()


def install_fake_metal():
    m = types.ModuleType("Metal")
    m.MTLResourceStorageModeShared = 0
    m.MTLSizeMake = lambda *a: a
    m.MTLCreateSystemDefaultDevice = lambda: None
    sys.modules["Metal"] = m


def make_runner():
    from tests.conftest import MetalKernelRunner  # the reference's runner

    class Runner(MetalKernelRunner):
        def __init__(self):
            self.device = FakeDevice()
            self.queue = FakeQueue()

        def compile(self, msl, name):
            return (name, msl)

        def load(self, path, name):
            return Pipeline(name, path[1])

    return Runner()


def run_reference_test(fn):
    """Run one reference test; capture its `expected` list if it makes one."""
    captured = {}

    def tracer(frame, event, arg):
        if event == "return" and frame.f_code is fn.__code__:
            exp = frame.f_locals.get("expected")
            if isinstance(exp, list):
                captured["expected"] = np.asarray(exp, dtype=np.float64)
        return tracer if frame.f_code is fn.__code__ else None

    sys.settrace(lambda f, e, a: tracer if f.f_code is fn.__code__ else None)
    try:
        fn(make_runner())
        ok, err = True, ""
    except AssertionError as e:  # the reference test rejected the oracle
        ok, err = False, str(e)
    finally:
        sys.settrace(None)
    return ok, err, captured.get("expected")


REFERENCE_TESTS = [
    # (test name in tests/test_emitter.py, file:line)
    ("test_int4_matmul", "tests/test_emitter.py:3009"),
    ("test_int4_matmul_gpu", "tests/test_emitter.py:6157"),
    ("test_int8_matmul", "tests/test_emitter.py:2576"),
    ("test_int8_matmul_gpu", "tests/test_emitter.py:6101"),
    ("test_flash_attention_single_head", "tests/test_emitter.py:1849"),
    ("test_flash_attention_multi_block", "tests/test_emitter.py:1926"),
    ("test_flash_attention_causal", "tests/test_emitter.py:2291"),
    ("test_flash_attention_gpu", "tests/test_emitter.py:5579"),
    ("test_causal_attention_gpu", "tests/test_emitter.py:5505"),
    ("test_gqa_attention", "tests/test_emitter.py:2482"),
    ("test_gqa_attention_gpu", "tests/test_emitter.py:5717"),
    ("test_kv_cache_attention", "tests/test_emitter.py:2124"),
    ("test_kv_cache_attention_gpu", "tests/test_emitter.py:5652"),
    ("test_batched_kv_decode", "tests/test_emitter.py:2908"),
    ("test_paged_attention", "tests/test_emitter.py:3188"),
    ("test_paged_attention_partial_page", "tests/test_emitter.py:3283"),
    ("test_paged_attention_gpu", "tests/test_emitter.py:5786"),
    ("test_multi_head_paged_attention", "tests/test_emitter.py:3710"),
    ("test_fp16_kv_attention", "tests/test_emitter.py:3809"),
    ("test_sliding_window_attention", "tests/test_emitter.py:3933"),
    ("test_sliding_window_attention_gpu", "tests/test_emitter.py:5866"),
    ("test_rope_attention", "tests/test_emitter.py:3088"),
    ("test_repeat_kv", "tests/test_emitter.py:4006"),
]

TRITON_FA_SHAPES = {
    False: [(1, 1, 32, 32), (1, 1, 64, 32), (1, 1, 64, 64), (1, 2, 64, 32), (2, 2, 64, 32), (1, 1, 128, 32)],
    True: [(1, 1, 32, 32), (1, 1, 64, 32), (1, 1, 64, 64), (1, 2, 64, 32), (1, 1, 128, 32)],
}  # tests/test_flash_attention.py:124-131 and :158-164


def _save(name, arrays):
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **arrays)
    return path


def main():
    install_fake_metal()
    sys.path.insert(0, REF)
    import importlib
    te = importlib.import_module("tests.test_emitter")
    manifest = {"reference_tests": [], "triton_fa": []}
    for tname, cite in REFERENCE_TESTS:
        DISPATCHES.clear()
        ok, err, expected = run_reference_test(getattr(te, tname))
        assert len(DISPATCHES) == 1, (tname, len(DISPATCHES))
        rec = dict(DISPATCHES[0])
        arrays = {k: np.asarray(v) for k, v in rec.items() if isinstance(v, np.ndarray)}
        meta = {k: v for k, v in rec.items() if not isinstance(v, np.ndarray)}
        if expected is not None:
            arrays["expected"] = expected
        _save("ref_" + tname, arrays)
        manifest["reference_tests"].append(
            {"test": tname, "cite": cite, "reference_test_passed": ok, "error": err,
             "has_expected": expected is not None, **meta})
        print(f"{tname:40s} reference assertions {'PASS' if ok else 'FAIL ' + err[:80]}")

    import torch
    tfa = importlib.import_module("tests.test_flash_attention")
    for causal, shapes in TRITON_FA_SHAPES.items():
        for (Z, H, N, D) in shapes:
            torch.manual_seed(42)
            q = torch.randn(Z, H, N, D, dtype=torch.float32)
            k = torch.randn(Z, H, N, D, dtype=torch.float32)
            v = torch.randn(Z, H, N, D, dtype=torch.float32)
            ref = tfa._ref_attention(q, k, v, causal=causal)
            name = f"triton_fa_{'causal' if causal else 'noncausal'}_{Z}x{H}x{N}x{D}"
            _save(name, {"q": q.numpy(), "k": k.numpy(), "v": v.numpy(), "out": ref.numpy()})
            manifest["triton_fa"].append({"name": name, "causal": causal, "shape": [Z, H, N, D],
                                          "cite": "tests/test_flash_attention.py:107-118"})
    manifest["kda"] = kda_goldens()
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)


KDA_CASES = [  # (name, B, T, H, D, with_initial_state, seed)
    ("kda_b1_t128_h1", 1, 128, 1, 128, False, 1),
    ("kda_b2_t64_h2_init", 2, 64, 2, 128, True, 2),
]


def kda_goldens():
    """KDA has no reference code (triton-metal ships none).  Golden vectors
    come from flash-linear-attention 0.5.1, fla.ops.kda.naive
    (naive_recurrent_kda), on inputs drawn as in oracle/kda.py.make_inputs."""
    import torch
    from fla.ops.kda.naive import naive_recurrent_kda
    from oracle import kda as okda
    out = []
    for name, B, T, H, D, init, seed in KDA_CASES:
        q, k, v, g, beta = okda.make_inputs(B, T, H, D, seed=seed)
        s0 = np.random.default_rng(seed + 100).standard_normal((B, H, D, D)) * 0.1 if init else None
        tt = lambda a: torch.tensor(a, dtype=torch.float32)
        o, S = naive_recurrent_kda(tt(q), tt(k), tt(v), tt(g), tt(beta), scale=None,
                                   initial_state=None if s0 is None else tt(s0), output_final_state=True)
        arrays = {"q": q.astype(np.float32), "k": k.astype(np.float32), "v": v.astype(np.float32),
                  "g": g.astype(np.float32), "beta": beta.astype(np.float32),
                  "o": o.numpy(), "S": S.numpy()}
        if s0 is not None:
            arrays["s0"] = s0.astype(np.float32)
        _save(name, arrays)
        out.append({"name": name, "B": B, "T": T, "H": H, "D": D, "initial_state": init,
                    "source": "fla 0.5.1 fla.ops.kda.naive.naive_recurrent_kda"})
    return out


if __name__ == "__main__":
    main()

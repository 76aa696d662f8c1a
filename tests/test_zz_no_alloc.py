"""The allocation-free KDA entry point, b2_kda_fwd_noalloc.

It exists for callers that cannot allocate device memory when they run KDA
(for example code running inside a custom allocator or memory pool that must
not be re-entered, or a plugin host that only hands over the input and output
buffers); it keeps its workspace in a fixed device array inside libb2.so.
These tests call it through the C ABI twice in a row and compare each result
with the regular entry point b2_kda_fwd (caller-provided workspace) at the
KDA tolerance, element-wise |x - ref| <= 2e-2 + 2e-2 |ref|.  This file is
collected last so that a run stopping at the first failure has already run
every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import kda as okda

pytestmark = pytest.mark.gpu
TOL = 2e-2


_DT = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}


def _inputs(cuda, B, T, H, seed, dtype=torch.bfloat16):
    q, k, v, g, beta = okda.make_inputs(B, T, H, 128, seed=seed)
    cv = lambda a: torch.tensor(a, dtype=dtype, device=cuda).contiguous()
    return cv(q), cv(k), cv(v), torch.tensor(g, dtype=torch.float32, device=cuda).contiguous(), cv(beta)


def _call(lib, name, q, k, v, g, beta, o, s_out, ws=None, s0=None):
    B, T, H, D = q.shape
    stream = torch.cuda.current_stream().cuda_stream
    args = [q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(),
            None if s0 is None else s0.data_ptr(), o.data_ptr(), s_out.data_ptr()]
    if ws is not None:
        args.append(ws.data_ptr())
    args += [B, T, H, D, D, 64, ctypes.c_float(D ** -0.5), _DT[q.dtype], stream]
    return getattr(lib, name)(*args)


def _close(x, ref):
    x, ref = x.double(), ref.double()
    err = (x - ref).abs()
    assert bool((err <= TOL + TOL * ref.abs()).all()), f"max err {err.max().item():.4g}"


def test_noalloc_matches_regular_entry_point_twice(cuda):
    from b200kern import _lib
    from b200kern.kda import workspace_size
    lib = _lib.load()
    for call, (B, T, H, seed) in enumerate([(1, 1024, 4, 5), (2, 512, 3, 6)]):
        q, k, v, g, beta = _inputs(cuda, B, T, H, seed)
        o_ref = torch.empty_like(v)
        s_ref = torch.empty(B, H, 128, 128, dtype=torch.float32, device=cuda)
        ws = torch.empty(workspace_size(B, T, H), dtype=torch.uint8, device=cuda)
        assert _call(lib, "b2_kda_fwd", q, k, v, g, beta, o_ref, s_ref, ws) == 0, lib.b2_last_error()
        o = torch.full_like(v, float("nan"))
        s = torch.full((B, H, 128, 128), float("nan"), dtype=torch.float32, device=cuda)
        st = _call(lib, "b2_kda_fwd_noalloc", q, k, v, g, beta, o, s)
        assert st == 0, lib.b2_last_error()
        torch.cuda.synchronize()
        _close(o, o_ref)
        _close(s, s_ref)


def test_noalloc_initial_state_and_fp16(cuda):
    """A non-zero fp32 initial state and fp16 operands, right after calls that
    left other contents in the shared device array."""
    from b200kern import _lib
    from b200kern.kda import workspace_size
    lib = _lib.load()
    B, T, H = 1, 768, 2
    q, k, v, g, beta = _inputs(cuda, B, T, H, 11, dtype=torch.float16)
    gen = torch.Generator().manual_seed(12)
    s0 = (torch.randn(B, H, 128, 128, generator=gen) * 0.3).to(cuda)
    o_ref = torch.empty_like(v)
    s_ref = torch.empty(B, H, 128, 128, dtype=torch.float32, device=cuda)
    ws = torch.empty(workspace_size(B, T, H), dtype=torch.uint8, device=cuda)
    assert _call(lib, "b2_kda_fwd", q, k, v, g, beta, o_ref, s_ref, ws, s0=s0) == 0, lib.b2_last_error()
    for _ in range(2):
        o = torch.full_like(v, float("nan"))
        s = torch.full((B, H, 128, 128), float("nan"), dtype=torch.float32, device=cuda)
        assert _call(lib, "b2_kda_fwd_noalloc", q, k, v, g, beta, o, s, s0=s0) == 0, lib.b2_last_error()
        torch.cuda.synchronize()
        _close(o, o_ref)
        _close(s, s_ref)


def test_noalloc_rejects_oversized_problem(cuda):
    from b200kern import _lib
    lib = _lib.load()
    q, k, v, g, beta = _inputs(cuda, 1, 64, 1, 0)
    # 1 x 16384 x 32 needs 8192 chunk-heads of workspace, above the 834 the array holds
    st = lib.b2_kda_fwd_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(), None,
                                v.data_ptr(), None, 1, 16384, 32, 128, 128, 64, ctypes.c_float(0.088), 1,
                                torch.cuda.current_stream().cuda_stream)
    assert st == -1
    assert b"exceeds" in lib.b2_last_error()

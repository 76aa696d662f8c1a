"""Host plan of the W4 decode GEMV, checked on CPU through b2_w4_gemv_plan.

The streaming kernel's consumer warp w waits on ring slot s % stages with
parity (s / stages) & 1; a parity wait one phase ahead returns at once, so a
slot must only ever be reused by the warp that waited on it before: the ring
holds a multiple of the 8 stage lanes (or one slot per group).  These tests
sweep shapes and SM counts and check that invariant, the TMA box limits, the
shared-memory budget and that the CTA slabs tile N exactly."""
import ctypes

import pytest

from b200kern import _lib

STAGE_LANES = 8
BUDGET = {1: 110 * 1024, 2: 227 * 1024}  # M <= 8: two CTAs per SM (PDL overlap); M <= 16: one


def _plan(M, N, K, G, zeros, sms):
    info = (ctypes.c_int64 * 6)()
    st = _lib.load().b2_w4_gemv_plan(M, N, K, G, int(zeros), sms, info)
    return st, list(info)


@pytest.mark.parametrize("sms", [148, 132, 20])
@pytest.mark.parametrize("M", [1, 8, 9, 16])
@pytest.mark.parametrize("zeros", [False, True])
def test_plan_invariants(M, zeros, sms):
    checked = 0
    for G in (32, 64, 128, 256):
        for K in (G, 2 * G, 1024, 4096, 8192, 14336, 28672):
            if K % G:
                continue
            for N in (8, 64, 1000, 4096, 11008, 14336, 20000, 65536):
                st, (grid, base, rem, stages, gps, smem) = _plan(M, N, K, G, zeros, sms)
                if st != 0:
                    assert st == -4, (M, N, K, G, st)  # unsupported -> generic kernel
                    continue
                checked += 1
                ngroups, rows = K // G, G // 8
                nt = 1 if M <= 8 else 2
                # CTA slabs tile the N / 8 column granules exactly, <= 128 columns each
                assert base * grid + rem == N // 8 and 0 <= rem < grid
                assert (base + (1 if rem else 0)) * 8 <= 128
                # ring-slot ownership (parity aliasing rule)
                assert 1 <= stages
                assert stages == ngroups or stages % STAGE_LANES == 0, (stages, ngroups)
                # one TMA box of gps groups fills gps consecutive slots
                assert gps in (1, 2, 4) and stages % gps == 0 and ngroups % gps == 0
                assert rows * gps <= 256 and ngroups <= 256  # TMA box dimensions
                assert 0 < smem <= BUDGET[nt]
    assert checked > 20


def test_plan_c1_shape():
    """The C1 decode shape on a 148-SM B200: one CTA per SM, 72/80-column
    slabs, a 16-slot ring in boxes of four groups (20 KB)."""
    st, (grid, base, rem, stages, gps, smem) = _plan(1, 11008, 4096, 128, False, 148)
    assert st == 0
    assert grid == 148 and base == 9 and rem == 1376 - 9 * 148
    assert stages == 16 and gps == 4
    assert smem <= 110 * 1024


def test_plan_rejects_unsupported_shapes():
    assert _plan(17, 11008, 4096, 128, False, 148)[0] == -4  # M > 16: GEMM path
    assert _plan(1, 11004, 4096, 128, False, 148)[0] == -4   # N % 8
    assert _plan(1, 4096, 4096, 96, False, 148)[0] == -4     # G not 32 x 2^k

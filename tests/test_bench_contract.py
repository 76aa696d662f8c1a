"""The bench's workload table and algorithmic-byte figures (no GPU).

Checks the numbers the roofline lines divide by: the W4 GEMV bytes per
launch match the C1 formula, each workload names its unit and bound,
and every committed ncu traffic figure belongs to a real workload."""
import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_contract_mod", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    argv = sys.argv
    sys.argv = ["bench.py"]
    try:
        spec.loader.exec_module(mod)
    finally:
        sys.argv = argv
    return mod


def test_c1_bytes_formula(bench):
    # K/8 * N * 4 (packed) + K/G * N * 2 (scales) + M*K*2 (x) + M*N*2 (out)
    for m in (1, 4, 16):
        assert bench.w4_gemv_bytes(m) == 512 * 11008 * 4 + 32 * 11008 * 2 + m * 4096 * 2 + m * 11008 * 2
    assert bench.w4_gemv_bytes(1) == 23279104


def test_workloads_declare_unit_and_bound(bench):
    for name, cls in bench.WORKLOADS.items():
        assert cls.unit in ("GB/s", "TFLOP/s", "tokens/s"), name
        assert cls.bound in ("hbm", "tensor"), name


def test_traffic_figures_name_workloads(bench):
    names = {getattr(cls, "name", k) for k, cls in bench.WORKLOADS.items()}
    for key, val in bench.NCU_TRAFFIC.items():
        assert key in names, key
        assert val is None or val > 0


def test_fa_window_visible_pairs(bench):
    # brute force over small S: key j visible to query i iff i - W < j <= i
    for S in (1, 7, 64, 200):
        for W in (1, 3, 64, 199, 200, 500):
            want = sum(1 for i in range(S) for j in range(S) if i - W < j <= i)
            assert bench.fa_visible_pairs(S, W) == want, (S, W)
    # W >= S is plain causal (S (S + 1) / 2 pairs)
    assert bench.fa_visible_pairs(8192, 8192) == 8192 * 8193 // 2

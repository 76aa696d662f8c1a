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
    """Every `traffic[...]` figure in profiles/*.md names a bench workload."""
    names = set(bench.WORKLOADS)
    for key, val in bench.ncu_traffic().items():
        assert key.split()[0] in names, key
        assert val > 0


def test_run_samples_counts_returned_units(bench):
    calls = []
    rate, n, el = bench.run_samples(lambda i: calls.append(i) or 2.0, None, warmup=2, steps=5)
    assert n == 5 and len(calls) == 7 and calls[:2] == [0, 1]
    assert rate == pytest.approx(10.0 / el)


def test_reference_arm_config_matches_ours(bench):
    """Both arms print config_of(workload) built from the same constructor
    (the reference arm builds it without device tensors)."""
    wl = bench.make_workload("fa_c0", 0, device=False)
    assert bench.config_of(wl) == {"workload": "fa_c0 B=2 H=8 S=1024 D=64 causal=True fp32 scale=1/8"}
    wl = bench.make_workload("w4a16_gemv", 0, 1, device=False)
    assert bench.config_of(wl) == {"workload": "w4a16_gemv M=1 K=4096 N=11008 G=128"}


def test_fa_window_visible_pairs(bench):
    # brute force over small S: key j visible to query i iff i - W < j <= i
    for S in (1, 7, 64, 200):
        for W in (1, 3, 64, 199, 200, 500):
            want = sum(1 for i in range(S) for j in range(S) if i - W < j <= i)
            assert bench.fa_visible_pairs(S, W) == want, (S, W)
    # W >= S is plain causal (S (S + 1) / 2 pairs)
    assert bench.fa_visible_pairs(8192, 8192) == 8192 * 8193 // 2

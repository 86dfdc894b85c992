"""bench.py's host-side arithmetic, without a GPU: the FLOP convention and the
per-configuration totals the measurement plan states, the algorithmic work each
kernel's roofline divides by, the workload shapes against BASELINE.json's
configurations, and the peak and traffic files the JSON line reads."""
import json
import os

import pytest

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("workload,fwd_gflop,step_gflop", [
    ("C1", 8.59, 30.1),            # (1,16,2048,64) causal
    ("C2", 34.4, 120.3),           # (1,8,4096,128) causal
    ("north_star", 550.0, 1924.4),  # (1,32,8192,128) causal
    ("C5", 140.7e3, 492.6e3),      # (1,32,131072,128) causal, before sharding
])
def test_flop_convention(workload, fwd_gflop, step_gflop):
    """fwd = 4*B*Hq*D*pairs with N(N+1)/2 causal pairs, fwd+bwd = 3.5 x fwd."""
    B, Hq, Hkv, N, D, causal, _ = bench.WORKLOADS[workload]
    assert bench.flops_fwd(B, Hq, N, D, causal) / 1e9 == pytest.approx(fwd_gflop, rel=2e-3)
    assert bench.step_flops(workload) / 1e9 == pytest.approx(step_gflop, rel=2e-3)


def test_noncausal_counts_every_pair():
    assert bench.flops_fwd(1, 1, 1000, 64, False) == 4.0 * 64 * 1000 * 1000
    assert bench.flops_fwd(1, 1, 1000, 64, True) == 4.0 * 64 * 1000 * 1001 / 2


def test_kernel_work_units():
    args = (4, 32, 8, 3000, 128, True)
    ff = bench.flops_fwd(4, 32, 3000, 128, True)
    assert bench.kernel_work("fwd", *args) == (ff, "TFLOP/s", "tensor")
    assert bench.kernel_work("bwd_fused", *args) == (2.5 * ff, "TFLOP/s", "tensor")
    assert bench.kernel_work("bwd_dkdv", *args)[0] == 2.0 * ff
    assert bench.kernel_work("bwd_dq", *args)[0] == 0.5 * ff
    # row sums: O and dO read, two fp32 row values written, the fp32 dq zeroed
    rows = 4 * 32 * 3000
    work, unit, bound = bench.kernel_work("bwd_rowsum", *args)
    assert (unit, bound) == ("GB/s", "hbm")
    assert work == 2 * rows * 128 * 2 + 2 * rows * 4 + rows * 128 * 4


def test_workloads_match_the_baseline_configs():
    configs = json.load(open(os.path.join(ROOT, "BASELINE.json")))["configs"]
    # configs 1, 2 and 5 quote one shape each; config 3 quotes (a) and (b)
    assert "B=1, Hq=Hkv=16, N=2048, D=64" in configs[0]
    assert bench.WORKLOADS["C1"][:5] == (1, 16, 16, 2048, 64)
    assert bench.WORKLOADS["C2"][:5] == (1, 8, 8, 4096, 128)
    assert "Hq=Hkv=8, N=4096, D=128" in configs[1]
    assert "B=4, Hq=32, Hkv=8, N=3000, D=128" in configs[2]
    assert "B=2, Hq=16, Hkv=1, N=1537, D=64" in configs[2]
    assert bench.WORKLOADS["C3a"][:5] == (4, 32, 8, 3000, 128)
    assert bench.WORKLOADS["C3b"][:5] == (2, 16, 1, 1537, 64)
    assert bench.WORKLOADS["C3a"][6] == 0.5 and bench.WORKLOADS["C3b"][6] == 0.5   # "x0.5"
    assert "B=1, Hq=32, Hkv=8, N=131072, D=128" in configs[4]
    assert bench.WORKLOADS["C5"][:5] == (1, 32, 8, 131072, 128)
    assert all(bench.WORKLOADS[w][5] for w in ("C1", "C2", "C3a", "C5", "north_star"))


def test_peak_and_traffic_files():
    tf, gbs, src = bench.load_peak()
    if os.path.exists(os.path.join(ROOT, "MEASURED_PEAKS.json")):
        pk = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        assert (tf, gbs) == (pk["bf16_tflops"], pk["hbm_gbs"]) and src.startswith("measured")
    else:
        assert src == "fallback"
    # the headline's fused-backward traffic comes from a committed ncu capture
    assert bench.load_traffic("C3a")["bwd_fused"] > 0
    assert bench.load_traffic("no such workload") == {}

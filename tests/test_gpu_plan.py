"""The fused backward's schedule query (fa_b200_backward_plan) on a B200: the
split it reports needs the GQA workspace, divides the group, and is the one the
backward runs (the split path's results are checked against the oracle by the
configuration tests, C3a non-causal and C3b among them)."""
import ctypes

import pytest

import _lib

pytestmark = pytest.mark.gpu


def plan(B, Hq, Hkv, N, D, causal, ws):
    g, h = ctypes.c_int(0), ctypes.c_int(0)
    st = _lib.lib().fa_b200_backward_plan(B, Hq, Hkv, N, D, int(causal), ws, ctypes.byref(g),
                                          ctypes.byref(h))
    assert st == 0, _lib.status_string(st)
    return g.value, h.value


@pytest.mark.parametrize("shape", [(4, 32, 8, 3000, 128, False), (4, 32, 8, 3000, 128, True),
                                   (2, 16, 1, 1537, 64, True), (1, 16, 8, 8192, 128, True),
                                   (1, 32, 32, 8192, 128, True)])
def test_plan_is_consistent(cuda, shape):
    B, Hq, Hkv, N, D, causal = shape
    lib = _lib.lib()
    group = Hq // Hkv
    gsplit, hg = plan(B, Hq, Hkv, N, D, causal, lib.fa_b200_backward_workspace_bytes_gqa(B, Hq, Hkv, N, D))
    assert 1 <= gsplit <= group and group % gsplit == 0
    assert 1 <= hg <= B * Hkv
    # without room for the fp32 dK/dV accumulators the group is never split
    gs0, hg0 = plan(B, Hq, Hkv, N, D, causal, lib.fa_b200_backward_workspace_bytes(B, Hq, N))
    assert gs0 == 1 and 1 <= hg0 <= B * Hkv
    if Hq == Hkv:
        assert gsplit == 1


def test_small_mqa_grid_splits(cuda):
    lib = _lib.lib()
    ws = lib.fa_b200_backward_workspace_bytes_gqa(2, 16, 1, 1537, 64)
    assert plan(2, 16, 1, 1537, 64, False, ws)[0] > 1

"""The no-allocation backward, fa_b200_backward_noalloc.

Some callers cannot give this library device memory of its own: their device
memory belongs to another allocator, or they must never call cudaMalloc on the
hot path. For them the backward keeps its Dv row sums in a fixed array compiled
into the library. This checks, through the C ABI, that two calls in a row (of
different shapes, so the second call finds the first one's leftovers in that
array) give the same dq, dk and dv as fa_b200_backward with a caller-provided
workspace -- on the fused path (fp32 dq) and on the deterministic one (fp16
dq, whose dK/dV and dQ kernels both read the array) -- that one case meets the
CPU oracle, and that sizes beyond the array are refused with a clear status.

The file is named to be collected last, so a run that stops at its first
failure has already run every other test.
"""
import pytest
import torch

import _lib
from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu

GRAD_FROB = 1e-2   # the gradient tolerance the parity tests use


def _both(cuda, B, Hq, Hkv, N, D, causal, seed, dq_fp32=1):
    """The same backward through fa_b200_backward (a caller workspace holding
    the per-row values only, so a GQA group is never split over CTAs) and
    through fa_b200_backward_noalloc, both into NaN-filled outputs. Returns
    (inputs, workspace result, no-allocation result)."""
    import fa_p100_ext
    lib = _lib.lib()
    host = orc.seeded_inputs(B, Hq, Hkv, N, D, seed=seed)
    q, k, v, do = (t.to(cuda) for t in host)
    o, lse = fa_p100_ext.forward(q, k, v, causal, False)
    stream = torch.cuda.current_stream().cuda_stream

    def outs():
        return (torch.full((B, Hq, N, D), float("nan"), device=cuda,
                           dtype=torch.float32 if dq_fp32 else torch.float16),
                torch.full_like(k, float("nan")), torch.full_like(v, float("nan")))

    ref = outs()
    ws_bytes = lib.fa_b200_backward_workspace_bytes(B, Hq, N)
    ws = torch.empty(ws_bytes // 4, device=cuda)
    st = lib.fa_b200_backward(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), o.data_ptr(),
                              lse.data_ptr(), ref[0].data_ptr(), dq_fp32, ref[1].data_ptr(),
                              ref[2].data_ptr(), ws.data_ptr(), ws_bytes, B, Hq, Hkv, N, D,
                              int(causal), stream)
    _lib.check(st, "fa_b200_backward")
    got = outs()
    st = lib.fa_b200_backward_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(),
                                      o.data_ptr(), lse.data_ptr(), got[0].data_ptr(), dq_fp32,
                                      got[1].data_ptr(), got[2].data_ptr(), B, Hq, Hkv, N, D,
                                      int(causal), stream)
    _lib.check(st, "fa_b200_backward_noalloc")
    torch.cuda.synchronize()
    assert _lib.device_error(0) == 0
    return host, ref, got


@pytest.mark.parametrize("dq_fp32", [1, 0], ids=["fused-fp32-dq", "deterministic-fp16-dq"])
def test_noalloc_matches_workspace_backward_twice(cuda, dq_fp32):
    """Two calls in a row, of different shapes (the second finds the first
    one's leftovers in the built-in array). dK/dV come from the same kernels
    reading the same row values, so they must match bit for bit; so must dQ on
    the deterministic path. The fused path adds dQ into fp32 in a run-dependent
    order, so there dQ is held to the tests' gradient tolerance."""
    calls = [(2, 8, 2, 777, 128, True, 3), (1, 4, 4, 300, 64, False, 4)]
    for B, Hq, Hkv, N, D, causal, seed in calls:
        _, ref, got = _both(cuda, B, Hq, Hkv, N, D, causal, seed, dq_fp32)
        for name, a, b in zip(("dq", "dk", "dv"), got, ref):
            assert torch.isfinite(a.float()).all(), f"{name} has unwritten entries"
            if name == "dq" and dq_fp32:
                err = orc.frob_rel(a, b)
                assert err <= GRAD_FROB, f"{name}: frobenius rel {err:.3e}"
            else:
                assert torch.equal(a, b), f"{name} differs from the workspace backward"


def test_noalloc_meets_the_oracle(cuda):
    """One GQA causal case through the no-allocation backward against the CPU
    oracle's analytic gradients."""
    (q, k, v, do), _, got = _both(cuda, 1, 8, 2, 333, 64, True, 9)
    rq, rk, rv = orc.attention_grads(q, k, v, do, True)
    for name, a, r in zip(("dq", "dk", "dv"), got, (rq, rk, rv)):
        err = orc.frob_rel(a, r)
        assert err <= GRAD_FROB, f"{name}: frobenius rel {err:.3e} against the oracle"


def test_noalloc_rejects_rows_beyond_scratch(cuda):
    lib = _lib.lib()
    max_rows = lib.fa_b200_backward_noalloc_max_rows()
    N = max_rows // 32 + 1            # 32 heads x N rows is one row over the limit
    dummy = torch.empty(16, device=cuda)
    p = dummy.data_ptr()
    st = lib.fa_b200_backward_noalloc(p, p, p, p, p, p, p, 1, p, p, 1, 32, 32, N, 64, 1,
                                      torch.cuda.current_stream().cuda_stream)
    assert st == 10   # FA_B200_ERR_SCRATCH_LIMIT, reported before any launch
    assert "exceeds the built-in scratch" in lib.fa_b200_last_error().decode()

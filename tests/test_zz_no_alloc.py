"""The no-allocation backward, fa_b200_backward_noalloc.

Some callers cannot give this library device memory of its own: their device
memory belongs to another allocator, or they must never call cudaMalloc on the
hot path. For them the backward keeps its Dv row sums in a fixed array compiled
into the library. This checks, through the C ABI, that two calls in a row (of
different shapes, so the second call finds the first one's leftovers in that
array) give the same dq, dk and dv as fa_b200_backward with a caller-provided
workspace, and that sizes beyond the array are refused with a clear status.

The file is named to be collected last, so a run that stops at its first
failure has already run every other test.
"""
import pytest
import torch

import _lib
from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu

GRAD_FROB = 1e-2   # the gradient tolerance the parity tests use


def _both(cuda, B, Hq, Hkv, N, D, causal, seed):
    import fa_p100_ext
    lib = _lib.lib()
    q, k, v, do = (t.to(cuda) for t in orc.seeded_inputs(B, Hq, Hkv, N, D, seed=seed))
    o, lse = fa_p100_ext.forward(q, k, v, causal, False)
    stream = torch.cuda.current_stream().cuda_stream

    def outs():
        return (torch.full((B, Hq, N, D), float("nan"), device=cuda),
                torch.full_like(k, float("nan")), torch.full_like(v, float("nan")))

    ref = outs()
    ws_bytes = lib.fa_b200_backward_workspace_bytes(B, Hq, N)
    ws = torch.empty(ws_bytes // 4, device=cuda)
    st = lib.fa_b200_backward(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), o.data_ptr(),
                              lse.data_ptr(), ref[0].data_ptr(), 1, ref[1].data_ptr(),
                              ref[2].data_ptr(), ws.data_ptr(), ws_bytes, B, Hq, Hkv, N, D,
                              int(causal), stream)
    _lib.check(st, "fa_b200_backward")
    got = outs()
    st = lib.fa_b200_backward_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(),
                                      o.data_ptr(), lse.data_ptr(), got[0].data_ptr(), 1,
                                      got[1].data_ptr(), got[2].data_ptr(), B, Hq, Hkv, N, D,
                                      int(causal), stream)
    _lib.check(st, "fa_b200_backward_noalloc")
    torch.cuda.synchronize()
    assert _lib.device_error(0) == 0
    return ref, got


def test_noalloc_matches_workspace_backward_twice(cuda):
    calls = [(2, 8, 2, 777, 128, True, 3), (1, 4, 4, 300, 64, False, 4)]
    for B, Hq, Hkv, N, D, causal, seed in calls:
        ref, got = _both(cuda, B, Hq, Hkv, N, D, causal, seed)
        for name, a, b in zip(("dq", "dk", "dv"), got, ref):
            assert torch.isfinite(a).all(), f"{name} has unwritten entries"
            err = orc.frob_rel(a, b)
            assert err <= GRAD_FROB, f"{name}: frobenius rel {err:.3e}"


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

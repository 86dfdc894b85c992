"""Layout self-test: one 128x128x128 tcgen05 MMA through the same TMA swizzle,
shared-memory descriptors and TMEM read-out the attention kernels use, against
torch.matmul in fp32. Isolates descriptor or swizzle errors from attention logic."""
import pytest
import torch

import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("a_mn,b_mn,a_threads", [(0, 0, 0), (0, 1, 0), (1, 1, 0), (1, 0, 0),
                                                 (0, 0, 1), (0, 1, 1), (0, 0, 2), (0, 1, 2)])
def test_selftest_gemm(cuda, a_mn, b_mn, a_threads):
    g = torch.Generator(device="cpu").manual_seed(1234 + 8 * a_mn + 4 * b_mn + a_threads)
    A = torch.randn(128, 128, generator=g).half()   # math A[m][k]
    Bm = torch.randn(128, 128, generator=g).half()  # math B[n][k]
    a_store = (A.t() if a_mn else A).contiguous().to(cuda)
    b_store = (Bm.t() if b_mn else Bm).contiguous().to(cuda)
    c = torch.full((128, 128), float("nan"), device=cuda)
    st = _lib.lib().fa_b200_selftest_gemm(a_store.data_ptr(), b_store.data_ptr(), c.data_ptr(),
                                          a_mn, b_mn, a_threads,
                                          torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "selftest")
    torch.cuda.synchronize()
    assert _lib.device_error(0) == 0
    ref = A.float() @ Bm.float().t()
    err = (c.cpu() - ref).abs().max().item()
    assert err < 1e-2, f"max abs err {err}"

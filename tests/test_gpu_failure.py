"""Failure detection on the GPU without a GPU fault: a bounded wait is made to
run out (a barrier that nothing arrives on, a 1 ms limit), and the error has to
surface on the host while the context stays usable.

fa_b200_selftest_wait runs the same bounded wait every kernel of the library
uses (mbar_wait_limit in csrc/sm100.cuh), with a short limit instead of the
production one second. The tests check that the wait gives up in about its
limit, that the device error word then reads FA_B200_DEVERR_SELFTEST, that the
product path raises RuntimeError (at once through check_device_errors, and at
the next op call through the asynchronous read every op enqueues), and that
the next normal call runs and matches the oracle with the word clear.
"""
import pytest
import torch

import _lib
from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu

DEVERR_SELFTEST = 6


def _timeout(limit_ns=1_000_000):
    """Runs the self-test wait; returns its CUDA-event duration in ms."""
    stream = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    _lib.check(_lib.lib().fa_b200_selftest_wait(limit_ns, stream.cuda_stream), "selftest_wait")
    b.record(stream)
    b.synchronize()
    return a.elapsed_time(b)


def _inputs(cuda):
    q, k, v, do = orc.seeded_inputs(1, 4, 2, 200, 64, seed=21)
    return (q, k, v, do), [t.to(cuda) for t in (q, k, v)]


def test_wait_runs_out_and_sets_the_error_word(cuda):
    import fa_p100
    fa_p100.check_device_errors(cuda)          # start clear
    ms = _timeout(1_000_000)
    assert 0.9 <= ms < 100.0, f"a 1 ms bounded wait took {ms:.3f} ms"
    assert _lib.device_error(0, reset=False) == DEVERR_SELFTEST
    with pytest.raises(RuntimeError, match="device error 6"):
        fa_p100.check_device_errors(cuda)
    assert _lib.device_error(0, reset=False) == 0   # the check cleared it


def test_product_path_raises_after_a_timeout_then_recovers(cuda):
    import fa_p100
    (q, k, v, do), dev_in = _inputs(cuda)
    fa_p100.flash_attn(*dev_in, True)            # the watch has a clean read pending
    torch.cuda.synchronize()
    _timeout(1_000_000)
    # the call after the timeout enqueues the read that sees the word ...
    fa_p100.flash_attn(*dev_in, True)
    torch.cuda.synchronize()
    # ... and the one after that raises, as AT_CUDA_CHECK would after a launch
    with pytest.raises(RuntimeError, match="device error 6"):
        fa_p100.flash_attn(*dev_in, True)
    assert _lib.device_error(0, reset=False) == 0
    # the context is usable and the next call is correct
    a = [t.clone().requires_grad_(True) for t in dev_in]
    o = fa_p100.flash_attn(*a, True)
    o.backward(do.to(cuda))
    fa_p100.check_device_errors(cuda)
    ro = orc.attention(q, k, v, True)
    rq, rk, rv = orc.attention_grads(q, k, v, do, True)
    assert orc.rel(o.detach(), ro) < 6e-2
    for x, r in zip(a, (rq, rk, rv)):
        assert orc.frob_rel(x.grad, r) < 1e-2

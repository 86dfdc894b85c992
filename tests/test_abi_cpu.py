"""The C ABI without a GPU: the library loads, exports every function
include/fa_b200.h declares, and rejects bad arguments with the documented status
codes before touching a device (so nothing here launches or needs CUDA)."""
import os
import re

import pytest

import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                      "include", "fa_b200.h")
P = 4096          # a 16-byte aligned fake device address, never dereferenced
MISALIGNED = 4097


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(fa_b200_\w+)\s*\(", text)))


def test_every_declared_symbol_is_exported():
    names = declared()
    assert len(names) >= 9
    lib = _lib.lib()
    for n in names:
        assert hasattr(lib, n), f"{n} declared in fa_b200.h but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def fwd(q=P, k=P, v=P, o=P, lse=P, B=1, Hq=4, Hkv=2, N=16, D=64):
    return _lib.lib().fa_b200_forward(q, k, v, o, lse, B, Hq, Hkv, N, D, 1, 0, None)


def test_forward_argument_errors():
    assert fwd(q=None) == 1
    assert fwd(lse=None) == 1
    assert fwd(D=96) == 2
    assert fwd(D=256) == 2
    assert fwd(N=0) == 3
    assert fwd(Hq=6, Hkv=4) == 3
    assert fwd(Hkv=0) == 3
    assert fwd(B=0) == 3
    assert fwd(o=MISALIGNED) == 4


def test_sequence_length_limit():
    # N above 2^30 is refused before any launch (padded row counts stay in int)
    assert fwd(N=(1 << 30) + 1) == 9
    lib = _lib.lib()
    assert lib.fa_b200_backward_workspace_bytes(1, 1, (1 << 30) + 1) == 0
    assert lib.fa_b200_backward_workspace_bytes(1, 1, 1 << 30) == 2 * 4 * (1 << 30)


def test_error_word_read_needs_a_buffer():
    assert _lib.lib().fa_b200_device_error_async(None, None) == 1


def bwd(ws=P, ws_bytes=1 << 20, stages=None, **kw):
    a = dict(B=1, Hq=4, Hkv=2, N=16, D=64)
    a.update(kw)
    lib = _lib.lib()
    args = [P, P, P, P, P, P, P, 1, P, P, ws, ws_bytes, a["B"], a["Hq"], a["Hkv"], a["N"],
            a["D"], 1]
    if stages is None:
        return lib.fa_b200_backward(*args, None)
    return lib.fa_b200_backward_stages(*args, stages, None)


def test_backward_argument_errors():
    assert bwd(D=80) == 2
    assert bwd(Hq=3, Hkv=2) == 3
    assert bwd(ws=None) == 7
    need = _lib.lib().fa_b200_backward_workspace_bytes(1, 4, 16)
    assert bwd(ws_bytes=need - 4) == 7             # one float short
    assert bwd(ws=MISALIGNED) == 4
    assert bwd(stages=16) == 3                      # unknown stage bit
    assert bwd(stages=8 | 2) == 3                   # FUSED excludes DKDV / DQ


def test_workspace_size():
    lib = _lib.lib()
    # Dv and LSE*log2e per row, each head padded to a multiple of 128 rows
    assert lib.fa_b200_backward_workspace_bytes(2, 8, 100) == 2 * 4 * 2 * 8 * 128
    assert lib.fa_b200_backward_workspace_bytes(1, 1, 129) == 2 * 4 * 256
    assert lib.fa_b200_backward_workspace_bytes(0, 1, 1) == 0


def test_noalloc_limit_and_errors():
    lib = _lib.lib()
    rows = lib.fa_b200_backward_noalloc_max_rows()
    assert rows == 1 << 21
    st = lib.fa_b200_backward_noalloc(P, P, P, P, P, P, P, 1, P, P, 1, 32, 32, rows // 32 + 1,
                                      64, 1, None)
    assert st == 10
    assert "exceeds the built-in scratch" in lib.fa_b200_last_error().decode()
    assert lib.fa_b200_backward_noalloc(None, P, P, P, P, P, P, 1, P, P, 1, 1, 1, 8, 64, 0,
                                        None) == 1


def test_release_build_has_no_tma_checks():
    """The release library answers the checked-build query with its own status
    (FA_B200_ERR_UNCHECKED_BUILD) and a zero word, touching no device; the
    checked library is a separate file, loaded with FA_B200_DEBUG=1."""
    import ctypes
    import _build
    if _build.checked_requested():
        pytest.skip("this process loaded the checked library")
    word = ctypes.c_ulonglong(7)
    assert _lib.lib().fa_b200_debug_tma_check(0, ctypes.byref(word), 1) == 12
    assert word.value == 0
    assert _lib.lib().fa_b200_debug_tma_check(0, None, 1) == 1
    assert os.path.basename(_lib.loaded_path()) == "libfa_b200.so"


def test_selftest_rejects_unsupported_mode():
    assert _lib.lib().fa_b200_selftest_gemm(P, P, P, 1, 0, 1, None) == 3


@pytest.mark.parametrize("code", range(0, 13))
def test_status_strings(code):
    text = _lib.status_string(code)
    assert text and text != "unknown status"
    assert _lib.status_string(99) == "unknown status"


def S(b=4 * 16 * 64, h=16 * 64, n=64):
    return _lib.Strides(b, h, n)


def fwd_strided(sq=None, so=None, o=P, D=64, dtype=0):
    lib = _lib.lib()
    sq = sq or S()
    return lib.fa_b200_forward_strided(P, sq, P, S(2 * 16 * 64), P, S(2 * 16 * 64), o, so or S(),
                                       P, 1, 4, 2, 16, D, dtype, 1, 0, None)


def test_strided_forward_argument_errors():
    # strides must be non-negative multiples of 16 bytes (8 fp16 elements)
    assert fwd_strided(sq=S(n=68)) == 4
    assert fwd_strided(sq=S(h=-64)) == 4
    assert fwd_strided(so=S(b=4 * 16 * 64 + 4)) == 4
    assert fwd_strided(o=MISALIGNED) == 4
    assert fwd_strided(D=96) == 2
    assert fwd_strided(dtype=2) == 11      # FA_B200_ERR_DTYPE
    assert fwd_strided(dtype=-1) == 11


def bwd_strided(sdq=None, dq_fp32=1, stages=0, dtype=0):
    lib = _lib.lib()
    sq, skv = S(), S(2 * 16 * 64)
    return lib.fa_b200_backward_strided(
        P, sq, P, skv, P, skv, P, sq, P, sq, P, P, sdq or S(), dq_fp32, P, skv, P, skv,
        P, 1 << 20, 1, 4, 2, 16, 64, dtype, 1, stages, None)


def test_strided_backward_argument_errors():
    # an fp32 dq needs strides in multiples of 4 elements, fp16 ones of 8
    assert bwd_strided(sdq=S(n=66)) == 4
    assert bwd_strided(sdq=S(n=68), dq_fp32=0) == 4
    assert bwd_strided(stages=8, dq_fp32=0) == 3     # the fused stage needs an fp32 dq
    assert bwd_strided(stages=64) == 3
    assert bwd_strided(dtype=7) == 11
    # accumulating (stage 16) needs the fused stage and an fp32 dq
    assert bwd_strided(stages=16) == 3
    assert bwd_strided(stages=1 | 16) == 3
    assert bwd_strided(stages=1 | 8 | 16, dq_fp32=0) == 3


def merge(o=P, lse=P, op=P, lp=P, D=64, dtype=0, so=None, sop=None, B=1):
    lib = _lib.lib()
    return lib.fa_b200_merge_partial(o, so or S(), lse, S(), op, sop or S(), lp, S(), B, 4, 16, D,
                                     dtype, None)


def test_merge_partial_argument_errors():
    assert merge(o=None) == 1
    assert merge(lp=None) == 1
    assert merge(D=96) == 2
    assert merge(B=0) == 3
    assert merge(dtype=3) == 11
    assert merge(o=MISALIGNED) == 4
    assert merge(so=S(n=66)) == 4          # fp32 rows: strides in multiples of 4 floats
    assert merge(sop=S(n=68)) == 4         # 16-bit rows: multiples of 8 elements


def test_strides_of_layouts():
    import torch
    # (B, H, N, D) view of (B, N, H, D) storage, as attention layers produce it
    t = torch.empty(2, 8192, 16, 128, dtype=torch.float16).transpose(1, 2)
    st = _lib.strides_of(t)
    assert (st.batch, st.head, st.row) == (8192 * 16 * 128, 128, 16 * 128)
    # size-1 dimensions take the contiguous stride whatever torch reports
    t1 = torch.empty(1, 8192, 16, 128, dtype=torch.float16).transpose(1, 2)
    assert _lib.strides_of(t1).batch == 16 * 8192 * 128
    # a non-contiguous D axis or an unaligned row stride does not qualify
    assert _lib.strides_of(torch.empty(1, 2, 16, 64, dtype=torch.float16).transpose(2, 3)) is None
    assert _lib.strides_of(torch.empty(1, 2, 16, 68, dtype=torch.float16)[..., :64]) is None
    assert _lib.strides_of(torch.empty(1, 2, 16, 72, dtype=torch.float16)[..., :64]) is not None


def test_workspace_size_queries():
    """The workspace size queries (pure host arithmetic)."""
    lib = _lib.lib()
    rows = lib.fa_b200_backward_workspace_bytes(2, 16, 1537)
    assert rows == 2 * 4 * 2 * 16 * 1664
    # the GQA query adds fp32 dK and dV accumulators
    assert lib.fa_b200_backward_workspace_bytes_gqa(2, 16, 1, 1537, 64) == rows + 2 * 4 * 2 * 1 * 1537 * 64
    assert lib.fa_b200_backward_workspace_bytes_gqa(0, 16, 1, 1537, 64) == 0


def test_backward_plan_argument_errors():
    """fa_b200_backward_plan checks its outputs and the shape before it looks
    at a device."""
    import ctypes
    lib = _lib.lib()
    g, h = ctypes.c_int(0), ctypes.c_int(0)
    assert lib.fa_b200_backward_plan(1, 4, 2, 16, 64, 1, 0, None, ctypes.byref(h)) == 1
    assert lib.fa_b200_backward_plan(1, 4, 2, 16, 64, 1, 0, ctypes.byref(g), None) == 1
    assert lib.fa_b200_backward_plan(1, 4, 2, 16, 96, 1, 0, ctypes.byref(g), ctypes.byref(h)) == 2
    assert lib.fa_b200_backward_plan(1, 6, 4, 16, 64, 1, 0, ctypes.byref(g), ctypes.byref(h)) == 3
    assert lib.fa_b200_backward_plan(0, 4, 2, 16, 64, 1, 0, ctypes.byref(g), ctypes.byref(h)) == 3

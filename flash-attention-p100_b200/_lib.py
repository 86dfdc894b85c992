"""ctypes binding of the C ABI in include/fa_b200.h.

Loads libfa_b200.so from this directory (building it with nvcc first when it
is missing or stale, as the reference builds its extension on import,
fa_p100.py:21-28). There is no fallback: if the library cannot be built or
loaded, importing this module raises.
"""
import ctypes
import os

from _build import build, checked_requested, lib_path, up_to_date



class Strides(ctypes.Structure):
    """fa_b200_strides: element strides (batch, head, row) of a (B, H, N, D)
    tensor whose D axis is contiguous."""
    _fields_ = [("batch", ctypes.c_int64), ("head", ctypes.c_int64), ("row", ctypes.c_int64)]


# The symbols include/fa_b200.h declares, with their ctypes signatures.
_P = ctypes.c_void_p
_I = ctypes.c_int
_SZ = ctypes.c_size_t
_S = Strides
SIGNATURES = {
    "fa_b200_forward": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P]),
    "fa_b200_forward_strided": (_I, [_P, _S, _P, _S, _P, _S, _P, _S, _P,
                                     _I, _I, _I, _I, _I, _I, _I, _I, _P]),
    "fa_b200_merge_partial": (_I, [_P, _S, _P, _S, _P, _S, _P, _S, _I, _I, _I, _I, _I, _P]),
    "fa_b200_backward_strided": (_I, [_P, _S, _P, _S, _P, _S, _P, _S, _P, _S, _P,
                                      _P, _S, _I, _P, _S, _P, _S, _P, _SZ,
                                      _I, _I, _I, _I, _I, _I, _I, _I, _P]),
    "fa_b200_backward_workspace_bytes": (_SZ, [_I, _I, _I]),
    "fa_b200_backward_workspace_bytes_gqa": (_SZ, [_I, _I, _I, _I, _I]),
    "fa_b200_backward_plan": (_I, [_I, _I, _I, _I, _I, _I, _SZ, _P, _P]),
    "fa_b200_backward": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _SZ,
                              _I, _I, _I, _I, _I, _I, _P]),
    "fa_b200_backward_stages": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _SZ,
                                     _I, _I, _I, _I, _I, _I, _I, _P]),
    "fa_b200_backward_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _P, _P,
                                      _I, _I, _I, _I, _I, _I, _P]),
    "fa_b200_backward_noalloc_max_rows": (_SZ, []),
    "fa_b200_device_error": (_I, [_I, _I]),
    "fa_b200_device_error_async": (_I, [_P, _P]),
    "fa_b200_debug_tma_check": (_I, [_I, ctypes.POINTER(ctypes.c_ulonglong), _I]),
    "fa_b200_selftest_wait": (_I, [ctypes.c_longlong, _P]),
    "fa_b200_status_string": (ctypes.c_char_p, [_I]),
    "fa_b200_last_error": (ctypes.c_char_p, []),
    "fa_b200_selftest_gemm": (_I, [_P, _P, _P, _I, _I, _I, _P]),
}

# FA_B200_DTYPE_* of the 16-bit tensors of the strided entry points
DTYPE_FP16, DTYPE_BF16 = 0, 1

_lib = None


def lib():
    """The loaded library (built on first use when needed): the release build,
    or with FA_B200_DEBUG=1 the checked one (TMA coordinate checks,
    fa_b200_debug_tma_check)."""
    global _lib
    if _lib is None:
        if not up_to_date():
            build()
        handle = ctypes.CDLL(lib_path())
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def status_string(code):
    return lib().fa_b200_status_string(int(code)).decode()


def check(code, what):
    """Turn a non-zero status into the RuntimeError TORCH_CHECK would raise."""
    if code != 0:
        detail = lib().fa_b200_last_error().decode()
        raise RuntimeError(f"{what}: {status_string(code)} (status {code})"
                           + (f": {detail}" if detail else ""))


def strides_of(t):
    """fa_b200_strides of a (B, H, N, D) tensor with a contiguous D axis; None
    if the layout does not qualify (the caller then passes a contiguous copy).
    A stride of a size-1 dimension is never used to address anything and is
    replaced by the contiguous one, which always satisfies the 16-byte rule."""
    if t.dim() != 4 or t.stride(3) != 1 or t.data_ptr() % 16:
        return None
    unit = 16 // t.element_size()
    B, H, N, D = t.shape
    dense = (H * N * D, N * D, D)
    st = [dense[i] if t.size(i) == 1 else t.stride(i) for i in range(3)]
    if any(x < 0 or x % unit for x in st):
        return None
    return Strides(*st)


def device_error(device=0, reset=True):
    """Error word set by a kernel whose bounded wait timed out (0 = none)."""
    return lib().fa_b200_device_error(int(device), 1 if reset else 0)


def loaded_path():
    """Path of the library this process loads (release, or checked with
    FA_B200_DEBUG=1)."""
    return os.path.abspath(lib_path())


def tma_check_word(device=0, reset=True):
    """The checked build's first TMA coordinate / alignment violation on
    `device` (0 = none); RuntimeError from a release build."""
    word = ctypes.c_ulonglong(0)
    check(lib().fa_b200_debug_tma_check(int(device), ctypes.byref(word), 1 if reset else 0),
          "fa_b200_debug_tma_check")
    return word.value

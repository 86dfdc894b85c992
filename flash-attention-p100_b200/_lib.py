"""ctypes binding of the C ABI in include/fa_b200.h.

Loads libfa_b200.so from this directory (building it with nvcc first when it
is missing or stale, as the reference builds its extension on import,
fa_p100.py:21-28). There is no fallback: if the library cannot be built or
loaded, importing this module raises.
"""
import ctypes
import os

from _build import LIB_PATH, build, up_to_date

# The symbols include/fa_b200.h declares, with their ctypes signatures.
_P = ctypes.c_void_p
_I = ctypes.c_int
_SZ = ctypes.c_size_t
SIGNATURES = {
    "fa_b200_forward": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P]),
    "fa_b200_backward_workspace_bytes": (_SZ, [_I, _I, _I]),
    "fa_b200_backward": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _SZ,
                              _I, _I, _I, _I, _I, _I, _P]),
    "fa_b200_backward_stages": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _SZ,
                                     _I, _I, _I, _I, _I, _I, _I, _P]),
    "fa_b200_backward_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _P, _P,
                                      _I, _I, _I, _I, _I, _I, _P]),
    "fa_b200_backward_noalloc_max_rows": (_SZ, []),
    "fa_b200_device_error": (_I, [_I, _I]),
    "fa_b200_status_string": (ctypes.c_char_p, [_I]),
    "fa_b200_last_error": (ctypes.c_char_p, []),
    "fa_b200_selftest_gemm": (_I, [_P, _P, _P, _I, _I, _I, _P]),
}

_lib = None


def lib():
    """The loaded library (built on first use when needed)."""
    global _lib
    if _lib is None:
        if not up_to_date():
            build()
        handle = ctypes.CDLL(LIB_PATH)
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


def device_error(device=0, reset=True):
    """Error word set by a kernel whose bounded wait timed out (0 = none)."""
    return lib().fa_b200_device_error(int(device), 1 if reset else 0)


def lib_path():
    return os.path.abspath(LIB_PATH)

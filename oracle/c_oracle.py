"""ctypes access to the fp64 C oracles -- TEST INFRASTRUCTURE ONLY.

  liboracle_f64.so      this repo's restatement (oracle/attn_ref_f64.c)
  _ref/libref_f64.so    the reference's own fp64 oracles, compiled from its
                        sources (attention.cu:72-102, bwd.cu:20-105) by
                        `make -C oracle ref`; only present where the reference
                        tree was available at build time.
"""
import ctypes
import json
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_D = ctypes.POINTER(ctypes.c_double)
_U16 = ctypes.POINTER(ctypes.c_uint16)
_I = ctypes.c_int


def reference_tree():
    """The reference's source tree: $FA_REFERENCE_TREE, else BASELINE.json's
    `reference_path`; None when neither names an existing directory."""
    path = os.environ.get("FA_REFERENCE_TREE")
    if not path:
        try:
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                path = json.load(f).get("reference_path")
        except (OSError, ValueError):
            path = None
    return path if path and os.path.isdir(path) else None


def _make(target=None, ref=None):
    cmd = ["make", "-s", "-C", HERE] + ([target] if target else []) + ([f"REF={ref}"] if ref else [])
    subprocess.run(cmd, check=True, capture_output=True)


def load_ours():
    path = os.path.join(HERE, "liboracle_f64.so")
    if not os.path.exists(path):
        _make()
    lib = ctypes.CDLL(path)
    lib.oracle_fwd_f64.argtypes = [_D, _D, _D, _D, _D] + [_I] * 6
    lib.oracle_bwd_f64.argtypes = [_D] * 7 + [_I] * 6
    lib.oracle_loss_f64.argtypes = [_D] * 4 + [_I] * 7 + [ctypes.c_size_t, ctypes.c_double]
    lib.oracle_loss_f64.restype = ctypes.c_double
    return lib


def load_reference(tree=None):
    """The reference's own fp64 oracles, or None when they cannot be built here.
    `tree` is the reference's source tree (default: reference_tree())."""
    path = os.path.join(HERE, "_ref", "libref_f64.so")
    if not os.path.exists(path):
        tree = tree or reference_tree()
        if not tree:
            return None
        _make("ref", tree)
    lib = ctypes.CDLL(path)
    lib.ref_attention_f64.argtypes = [_U16, _U16, _U16, _D, _I, _I, _I, _I]
    lib.ref_bwd_f64.argtypes = [_U16] * 4 + [_D] * 3 + [_I] * 4
    lib.ref_loss_f64.argtypes = [_U16] * 4 + [_I] * 5 + [ctypes.c_size_t, ctypes.c_double]
    lib.ref_loss_f64.restype = ctypes.c_double
    return lib


def _dp(a):
    return a.ctypes.data_as(_D)


def _hp(a):
    return a.view(np.uint16).ctypes.data_as(_U16)


def f64(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float64))


def fwd(lib, q, k, v, causal):
    """O, LSE in fp64 from (B,Hq,N,D) / (B,Hkv,N,D) float arrays."""
    q, k, v = f64(q), f64(k), f64(v)
    B, Hq, N, D = q.shape
    o = np.empty_like(q)
    lse = np.empty((B, Hq, N))
    lib.oracle_fwd_f64(_dp(q), _dp(k), _dp(v), _dp(o), _dp(lse), B, Hq, k.shape[1], N, D,
                       int(causal))
    return o, lse


def bwd(lib, q, k, v, do, causal):
    q, k, v, do = f64(q), f64(k), f64(v), f64(do)
    B, Hq, N, D = q.shape
    dq, dk, dv = np.empty_like(q), np.empty_like(k), np.empty_like(v)
    lib.oracle_bwd_f64(_dp(q), _dp(k), _dp(v), _dp(do), _dp(dq), _dp(dk), _dp(dv), B, Hq,
                       k.shape[1], N, D, int(causal))
    return dq, dk, dv


def loss(lib, q, k, v, do, causal, which, idx, pert):
    q, k, v, do = f64(q), f64(k), f64(v), f64(do)
    B, Hq, N, D = q.shape
    return lib.oracle_loss_f64(_dp(q), _dp(k), _dp(v), _dp(do), B, Hq, k.shape[1], N, D,
                               int(causal), which, idx, pert)


def ref_fwd(lib, q16, k16, v16, causal):
    """The reference's attention_ref_f64 on fp16 arrays (BH, N, d), no GQA."""
    q16, k16, v16 = (np.ascontiguousarray(a, dtype=np.float16) for a in (q16, k16, v16))
    BH, N, d = q16.shape
    o = np.empty((BH, N, d))
    lib.ref_attention_f64(_hp(q16), _hp(k16), _hp(v16), _dp(o), BH, N, d, int(causal))
    return o


def ref_bwd(lib, q16, k16, v16, do16, causal):
    arrs = [np.ascontiguousarray(a, dtype=np.float16) for a in (q16, k16, v16, do16)]
    BH, N, d = arrs[0].shape
    dq, dk, dv = (np.empty((BH, N, d)) for _ in range(3))
    lib.ref_bwd_f64(*(_hp(a) for a in arrs), _dp(dq), _dp(dk), _dp(dv), BH, N, d, int(causal))
    return dq, dk, dv

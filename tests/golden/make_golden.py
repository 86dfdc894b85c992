"""Generate golden vectors from the reference's own Python oracle.

Run in a container that has the reference tree (it is not needed afterwards):

    python tests/golden/make_golden.py [/path/to/reference]

(default: $FA_REFERENCE_TREE, else the `reference_path` BASELINE.json names)

It imports the reference module fa_p100 (fa_p100.py) with only its JIT build of
the sm_60 extension stubbed out (torch.utils.cpp_extension.load, fa_p100.py:21-28,
cannot build or run without that GPU), and calls its `reference()` (fa_p100.py:65-75)
on fp32 copies of seeded fp16 inputs, so the returned O is the reference's fp32
result (its final `.to(q.dtype)` is then a no-op). dQ/dK/dV are autograd
gradients through that same function, as test_fa_p100.py:90-96 takes them. The
reference has no Python LSE; the LSE stored here is torch.logsumexp of the
scaled, causal-masked fp32 logits, the quantity its kernel writes
(flash_fwd.cuh:321-330).

Each case is one .npz: q, k, v, dO as fp16, and o, lse, dq, dk, dv as fp32.
"""
import importlib.util
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import c_oracle  # noqa: E402
from oracle.attention_oracle import seeded_inputs  # noqa: E402

# name: (B, Hq, Hkv, N, D, causal, seed, qk_scale)
CASES = {
    "mha_n7_d64": (1, 2, 2, 7, 64, False, 1, 1.0),
    "mha_n7_d64_causal": (1, 2, 2, 7, 64, True, 1, 1.0),
    "gqa_n65_d64_causal": (1, 4, 2, 65, 64, True, 2, 1.0),
    "mqa_n33_d128": (1, 4, 1, 33, 128, False, 3, 1.0),
    "mha_n1_d128_causal": (2, 2, 2, 1, 128, True, 4, 1.0),
    "regime_x10_n64_d64_causal": (1, 2, 2, 64, 64, True, 5, 10.0),
    "regime_x005_n40_d128": (1, 1, 1, 40, 128, False, 6, 0.05),
    "regime_x3_n48_d64": (1, 2, 1, 48, 64, False, 7, 3.0),
}


def import_reference(ref_dir):
    import torch.utils.cpp_extension as cpp_ext
    real_load = cpp_ext.load
    cpp_ext.load = lambda *a, **k: None   # the sm_60 extension is never built or used
    try:
        spec = importlib.util.spec_from_file_location("fa_p100_reference",
                                                      os.path.join(ref_dir, "fa_p100.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        cpp_ext.load = real_load
    return mod


def lse_of(q, k, causal):
    g = q.shape[1] // k.shape[1]
    kk = k.repeat_interleave(g, dim=1) if g > 1 else k
    s = (q @ kk.transpose(-1, -2)) * (1.0 / math.sqrt(q.shape[-1]))
    if causal:
        n = q.shape[-2]
        s = s.masked_fill(torch.ones(n, n, dtype=torch.bool).triu(1), float("-inf"))
    return torch.logsumexp(s, dim=-1)


def main(ref_dir=None):
    ref_dir = ref_dir or c_oracle.reference_tree()
    if not ref_dir:
        raise SystemExit("usage: make_golden.py <reference source tree> "
                         "(or set FA_REFERENCE_TREE)")
    ref = import_reference(ref_dir)
    for name, (B, Hq, Hkv, N, D, causal, seed, qs) in CASES.items():
        q, k, v, do = seeded_inputs(B, Hq, Hkv, N, D, seed=seed, qk_scale=qs)
        qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
        o = ref.reference(qf, kf, vf, causal)
        o.backward(do.float())
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            q=q.numpy(), k=k.numpy(), v=v.numpy(), dO=do.numpy(),
            o=o.detach().numpy(), lse=lse_of(qf.detach(), kf.detach(), causal).numpy(),
            dq=qf.grad.numpy(), dk=kf.grad.numpy(), dv=vf.grad.numpy(),
            meta=np.array([B, Hq, Hkv, N, D, int(causal), seed], dtype=np.int64),
            qk_scale=np.array(qs))
        print("wrote", name)


if __name__ == "__main__":
    main(*sys.argv[1:])

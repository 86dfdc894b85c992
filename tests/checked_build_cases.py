"""Child program of test_gpu_checked_build.py (not a test module itself).

Runs with FA_B200_DEBUG=1, so this process loads the checked library
(libfa_b200_debug.so, every TMA copy testing its coordinates and
shared-memory alignment first). It drives every kernel path on small shapes
against the CPU oracle -- forward (small-grid and persistent), fused and
deterministic backward, fp16 and bf16, MHA / GQA / MQA (the split group), N
from 1 to ragged thousands, D 64 and 128, strided (B, N, H, D) inputs, the
accumulating backward and the merge the ring uses, the no-allocation
backward -- and prints one JSON line: the failed cases, the TMA check word
and the device error word.
"""
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for _p in (os.path.join(ROOT, "flash-attention-p100_b200"), ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

import _lib  # noqa: E402
import fa_p100  # noqa: E402
import fa_p100_ext  # noqa: E402
from oracle import attention_oracle as orc  # noqa: E402

O_REL = 6e-2                                   # the reference's `rel` gate
GRAD_FROB = {torch.float16: 1e-2, torch.bfloat16: 2e-2}

dev = torch.device("cuda", 0)
failures = []
ran = 0


def fail(name, what):
    failures.append(f"{name}: {what}")


def check(name, got, ref, tol, metric=orc.frob_rel):
    """Relative error gate; an all-zero reference (dQ and dK of a one-key causal
    row: P = 1, so dS = P (dP - rowsum(dO o O)) = 0) is checked absolutely."""
    ref_f = torch.as_tensor(ref).detach().double().cpu()
    if ref_f.abs().max().item() < 1e-6:
        e = torch.as_tensor(got).detach().double().cpu().abs().max().item()
        if not (e < 1e-3):
            fail(name, f"max |got| {e:.3e} where the oracle is zero")
        return
    e = metric(got, ref)
    if not (e < tol):
        fail(name, f"error {e:.3e} >= {tol}")


def autograd_case(B, Hq, Hkv, N, D, causal, dtype=torch.float16, seed=0):
    """flash_attn forward + autograd backward (the fused kernel) vs the oracle."""
    global ran
    name = f"autograd {B}x{Hq}/{Hkv}x{N}x{D} causal={causal} {dtype}"
    host = [t.to(dtype) for t in orc.seeded_inputs(B, Hq, Hkv, N, D, seed=seed)]
    a = [t.to(dev).requires_grad_(True) for t in host[:3]]
    o = fa_p100.flash_attn(*a, causal)
    o.backward(host[3].to(dev))
    torch.cuda.synchronize()
    check(name + " O", o.detach(), orc.attention(*host[:3], causal), O_REL, orc.rel)
    refs = orc.attention_grads(*host, causal)
    for x, r, n in zip(a, refs, ("dq", "dk", "dv")):
        check(f"{name} {n}", x.grad, r, GRAD_FROB[dtype])
    ran += 1


def deterministic_case(B, Hq, Hkv, N, D, causal, seed=0):
    """The two-kernel backward (fp16 dq: dK/dV, then dQ) vs the oracle."""
    global ran
    name = f"deterministic {B}x{Hq}/{Hkv}x{N}x{D} causal={causal}"
    q, k, v, do = orc.seeded_inputs(B, Hq, Hkv, N, D, seed=seed)
    g = [t.to(dev) for t in (q, k, v, do)]
    o, lse = fa_p100_ext.forward(g[0], g[1], g[2], causal, False)
    dq, dk, dv = fa_p100_ext.backward_into(g[0], g[1], g[2], g[3], o, lse, causal,
                                           dq_dtype=torch.float16)
    torch.cuda.synchronize()
    for x, r, n in zip((dq, dk, dv), orc.attention_grads(q, k, v, do, causal), ("dq", "dk", "dv")):
        check(f"{name} {n}", x, r, GRAD_FROB[torch.float16])
    ran += 1


def strided_case(B, Hq, Hkv, N, D, causal, seed=0):
    """(B, N, H, D) storage read in place and O written in that layout."""
    global ran
    name = f"strided {B}x{Hq}/{Hkv}x{N}x{D} causal={causal}"
    q, k, v, do = orc.seeded_inputs(B, Hq, Hkv, N, D, seed=seed)
    bnhd = [t.transpose(1, 2).contiguous().to(dev).transpose(1, 2) for t in (q, k, v)]
    a = [t.detach().requires_grad_(True) for t in bnhd]
    o = fa_p100.flash_attn_bnhd(*a, causal=causal)          # (B, N, H, D)
    o.backward(do.transpose(1, 2).to(dev))
    torch.cuda.synchronize()
    check(name + " O", o.transpose(1, 2), orc.attention(q, k, v, causal), O_REL, orc.rel)
    for x, r, n in zip(a, orc.attention_grads(q, k, v, do, causal), ("dq", "dk", "dv")):
        check(f"{name} {n}", x.grad, r, GRAD_FROB[torch.float16])
    ran += 1


def ring_ops_case(B, Hq, Hkv, N, D, seed=0):
    """The accumulating backward (gradients added into fp32 dq, dk, dv) and the
    partial-result merge, the two calls a ring step makes, on one GPU: the
    first N/2 queries against the two halves of the keys (square pieces, as the
    ring's are), merged, then both pieces' gradients accumulated."""
    global ran
    name = f"ring ops {B}x{Hq}/{Hkv}x{N}x{D}"
    q, k, v, do = orc.seeded_inputs(B, Hq, Hkv, N, D, seed=seed)
    h = N // 2
    qh, doh = q[:, :, :h], do[:, :, :h]
    g = [t.to(dev) for t in (qh, k, v, doh)]
    halves = (slice(0, h), slice(h, N))
    parts = [fa_p100_ext.forward(g[0], g[1][:, :, s], g[2][:, :, s], False, False) for s in halves]
    o, lse = parts[0][0].float(), parts[0][1].clone()
    fa_p100_ext.merge_partial(o, lse, parts[1][0], parts[1][1])
    check(name + " merged O", o, orc.attention(qh, k, v, False), O_REL, orc.rel)
    o16 = o.half()
    dq = torch.zeros(qh.shape, device=dev)
    dk = torch.zeros(k.shape, device=dev)
    dv = torch.zeros(v.shape, device=dev)
    for s in halves:
        fa_p100_ext.backward_accumulate(g[0], g[1][:, :, s], g[2][:, :, s], g[3], o16, lse, False,
                                        dq, dk[:, :, s], dv[:, :, s])
    torch.cuda.synchronize()
    refs = orc.attention_grads(qh, k, v, doh, False)
    for x, r, n in zip((dq, dk, dv), refs, ("dq", "dk", "dv")):
        check(f"{name} {n}", x, r, GRAD_FROB[torch.float16])
    ran += 1


def noalloc_case(B, Hq, Hkv, N, D, causal, seed=0):
    """fa_b200_backward_noalloc (its row values in the library's own array)."""
    global ran
    name = f"noalloc {B}x{Hq}/{Hkv}x{N}x{D} causal={causal}"
    q, k, v, do = orc.seeded_inputs(B, Hq, Hkv, N, D, seed=seed)
    g = [t.to(dev) for t in (q, k, v, do)]
    o, lse = fa_p100_ext.forward(g[0], g[1], g[2], causal, False)
    dq = torch.empty(q.shape, device=dev)
    dk, dv = torch.empty_like(g[1]), torch.empty_like(g[2])
    st = _lib.lib().fa_b200_backward_noalloc(
        g[0].data_ptr(), g[1].data_ptr(), g[2].data_ptr(), g[3].data_ptr(), o.data_ptr(),
        lse.data_ptr(), dq.data_ptr(), 1, dk.data_ptr(), dv.data_ptr(), B, Hq, Hkv, N, D,
        1 if causal else 0, torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "fa_b200_backward_noalloc")
    torch.cuda.synchronize()
    for x, r, n in zip((dq, dk, dv), orc.attention_grads(q, k, v, do, causal), ("dq", "dk", "dv")):
        check(f"{name} {n}", x, r, GRAD_FROB[torch.float16])
    ran += 1


def main():
    if os.environ.get("FA_B200_DEBUG") != "1" or \
            os.path.basename(_lib.loaded_path()) != "libfa_b200_debug.so":
        raise SystemExit("run with FA_B200_DEBUG=1: this program checks the checked library")
    _lib.tma_check_word(0, reset=True)
    seed = 0
    for D in (64, 128):
        for (B, Hq, Hkv, N, causal) in ((1, 4, 2, 1, True), (1, 4, 4, 65, False),
                                        (2, 8, 2, 333, True), (1, 16, 1, 1023, True),
                                        (1, 8, 8, 2048, True), (4, 16, 4, 1000, True),
                                        (2, 16, 1, 1537, False)):
            seed += 1
            autograd_case(B, Hq, Hkv, N, D, causal, seed=seed)
        autograd_case(2, 8, 2, 333, D, True, dtype=torch.bfloat16, seed=100 + D)
        deterministic_case(2, 8, 2, 333, D, True, seed=200 + D)
        deterministic_case(1, 4, 4, 1000, D, False, seed=300 + D)
        strided_case(2, 8, 2, 515, D, True, seed=400 + D)
        ring_ops_case(1, 8, 2, 512, D, seed=500 + D)
        noalloc_case(1, 8, 2, 777, D, True, seed=600 + D)
    word = _lib.tma_check_word(0, reset=True)
    print(json.dumps({"cases": ran, "failures": failures, "tma_check": word,
                      "device_error": _lib.device_error(0)}))


if __name__ == "__main__":
    main()

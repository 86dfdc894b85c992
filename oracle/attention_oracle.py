"""CPU oracle for the attention hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import this module, and only as the checker or the timed CPU baseline;
the product path (flash-attention-p100_b200/) never does.

What it restates, from the reference (qr0n/flash-attention-p100):
  * `attention`      -- fa_p100.reference (fa_p100.py:65-75): GQA by repeating
                        K/V heads (fa_p100.py:58-62), fp32 logits q.k * 1/sqrt(D)
                        with the scale applied to the fp32 product, causal mask
                        j > i -> -inf, softmax, @ V. Returned in fp32 (no final
                        cast) so fp16 kernel output can be compared against it.
  * `lse`            -- m + ln(sum exp(s - m)) of the same masked fp32 logits;
                        the kernels' LSE convention (flash_fwd.cuh:321-330).
  * `attention_grads`-- the analytic gradients of bwd_ref_f64 (bwd.cu:20-69):
                        Dv = rowsum(dO o O), dS = P o (dO V^T - Dv),
                        dV = P^T dO, dK = scale dS^T Q, dQ = scale dS K, with
                        GQA gradients summed over the heads sharing a kv head.
  * `rel`            -- the regression metric max|got - ref| / rms(ref)
                        (test_fa_p100.py:35-37).
Parity is pinned by tests/test_oracle.py against golden vectors produced by the
reference's own `reference()` function (tests/golden/make_golden.py) and
against the reference's fp64 C++ oracle built from its sources (oracle/Makefile).

Memory is bounded by processing one (batch, query head) at a time, so the
full-size configurations run on a host without materialising B*H*N*N logits.
"""
import math

import numpy as np
import torch


def _group(q, k):
    hq, hkv = q.shape[1], k.shape[1]
    assert hq % hkv == 0
    return hq // hkv


def _scores(qh, kh, causal):
    """fp32 logits for one head: (N, N) = qh @ kh^T / sqrt(D), causal-masked."""
    d = qh.shape[-1]
    s = (qh @ kh.transpose(0, 1)) * (1.0 / math.sqrt(d))
    if causal:
        n = qh.shape[0]
        mask = torch.ones(n, n, dtype=torch.bool, device=qh.device).triu(1)
        s = s.masked_fill(mask, float("-inf"))
    return s


def _prep(tensors, device):
    # TF32 would round the fp32 products; the oracle must not.
    if torch.device(device).type == "cuda":
        torch.backends.cuda.matmul.allow_tf32 = False
    return [t.detach().to(device, torch.float32) for t in tensors]


def attention(q, k, v, causal=False, with_lse=False, device="cpu"):
    """O (B,Hq,N,D) fp32 [and LSE (B,Hq,N) fp32], computed in fp32 on `device`
    (the CPU by default; a GPU only for configurations too large for the host)."""
    q, k, v = _prep((q, k, v), device)
    B, Hq, N, D = q.shape
    g = _group(q, k)
    o = torch.empty(B, Hq, N, D, device=device)
    lse = torch.empty(B, Hq, N, device=device)
    for b in range(B):
        for h in range(Hq):
            s = _scores(q[b, h], k[b, h // g], causal)
            lse[b, h] = torch.logsumexp(s, dim=-1)
            o[b, h] = torch.softmax(s, dim=-1) @ v[b, h // g]
    return (o, lse) if with_lse else o


def attention_grads(q, k, v, do, causal=False, device="cpu"):
    """(dQ, dK, dV) in fp32 for loss = sum(dO o O), O = attention(q, k, v)."""
    q, k, v, do = _prep((q, k, v, do), device)
    B, Hq, N, D = q.shape
    g = _group(q, k)
    scale = 1.0 / math.sqrt(D)
    dq = torch.zeros_like(q)
    dk = torch.zeros_like(k)
    dv = torch.zeros_like(v)
    for b in range(B):
        for h in range(Hq):
            kh, vh = k[b, h // g], v[b, h // g]
            p = torch.softmax(_scores(q[b, h], kh, causal), dim=-1)
            oh = p @ vh
            dvec = (do[b, h] * oh).sum(-1, keepdim=True)
            ds = p * (do[b, h] @ vh.transpose(0, 1) - dvec)
            dq[b, h] = scale * (ds @ kh)
            dk[b, h // g] += scale * (ds.transpose(0, 1) @ q[b, h])
            dv[b, h // g] += p.transpose(0, 1) @ do[b, h]
    return dq, dk, dv


def rel(got, ref):
    """max|got - ref| / rms(ref), the reference's test metric (test_fa_p100.py:35-37)."""
    got = torch.as_tensor(got).detach().float().cpu()
    ref = torch.as_tensor(ref).detach().float().cpu()
    return ((got - ref).abs().max() / ref.pow(2).mean().sqrt()).item()


def frob_rel(got, ref):
    """||got - ref||_F / ||ref||_F."""
    got = torch.as_tensor(got).detach().double().cpu()
    ref = torch.as_tensor(ref).detach().double().cpu()
    return (torch.linalg.vector_norm(got - ref) / torch.linalg.vector_norm(ref)).item()


def seeded_inputs(B, Hq, Hkv, N, D, seed=0, scale=1.0, qk_scale=None, device="cpu"):
    """q, k, v, dO as fp16, i.i.d. N(0,1)*scale from one torch.Generator seed.
    `qk_scale` (if given) scales q and k only, as the reference's input regimes
    do (test_fa_p100.py:116-123)."""
    gen = torch.Generator(device="cpu").manual_seed(seed)
    qs = scale if qk_scale is None else qk_scale

    def draw(h, s):
        return (torch.randn(B, h, N, D, generator=gen) * s).half().to(device)

    q = draw(Hq, qs)
    k = draw(Hkv, qs)
    v = draw(Hkv, scale)
    do = draw(Hq, scale)
    return q, k, v, do


def flops_fwd(B, Hq, N, D, causal):
    """Algorithmic forward FLOPs: 4*B*Hq*D*P, P = N^2 or N(N+1)/2 causal pairs."""
    pairs = N * (N + 1) / 2 if causal else float(N) * N
    return 4.0 * B * Hq * D * pairs


def to_numpy(t):
    return np.ascontiguousarray(torch.as_tensor(t).detach().cpu().numpy())


def reference_step(q, k, v, do, causal=False):
    """One fwd+bwd of the reference's CPU path, timed as the CPU baseline:
    fa_p100.reference's formula (fa_p100.py:65-75) in fp32 on the host, with
    the gradients taken by autograd as the reference's tests take them
    (test_fa_p100.py:90-96). Returns (O, dQ, dK, dV)."""
    qf, kf, vf = (t.detach().to("cpu", torch.float32).requires_grad_(True) for t in (q, k, v))
    g = _group(qf, kf)
    ke = kf.repeat_interleave(g, dim=1) if g > 1 else kf
    ve = vf.repeat_interleave(g, dim=1) if g > 1 else vf
    s = (qf @ ke.transpose(-1, -2)) * (1.0 / math.sqrt(qf.shape[-1]))
    if causal:
        n = qf.shape[-2]
        s = s.masked_fill(torch.ones(n, n, dtype=torch.bool).triu(1), float("-inf"))
    o = torch.softmax(s, dim=-1) @ ve
    o.backward(do.detach().to("cpu", torch.float32))
    return o.detach(), qf.grad, kf.grad, vf.grad


def attention_grads_given_lse(q, k, v, do, o, lse, causal=False):
    """Backward of one attention piece given the softmax statistics of the
    whole row (what a ring step sees): P = exp(scale S - LSE), Dv = rowsum(dO o O),
    dS = P o (dO V^T - Dv), dQ = scale dS K, dK = scale dS^T Q, dV = P^T dO --
    the reference backward's formulas (flash_bwd.cuh:66-78, :267-281) with the
    forward's LSE passed in rather than recomputed. fp32, CPU, GQA-aware."""
    q, k, v, do, o = (t.detach().to("cpu", torch.float32) for t in (q, k, v, do, o))
    lse = lse.detach().to("cpu", torch.float32)
    B, Hq, N, D = q.shape
    g = _group(q, k)
    scale = 1.0 / math.sqrt(D)
    dq = torch.zeros_like(q)
    dk = torch.zeros_like(k)
    dv = torch.zeros_like(v)
    for b in range(B):
        for h in range(Hq):
            kh, vh = k[b, h // g], v[b, h // g]
            p = torch.exp(_scores(q[b, h], kh, causal) - lse[b, h][:, None])
            dvec = (do[b, h] * o[b, h]).sum(-1, keepdim=True)
            ds = p * (do[b, h] @ vh.transpose(0, 1) - dvec)
            dq[b, h] = scale * (ds @ kh)
            dk[b, h // g] += scale * (ds.transpose(0, 1) @ q[b, h])
            dv[b, h // g] += p.transpose(0, 1) @ do[b, h]
    return dq, dk, dv

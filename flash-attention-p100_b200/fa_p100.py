"""FlashAttention-2 for B200 (sm_100a) as a torch autograd Function.

Drop-in for the reference module of the same name (fa_p100.py): the same
`flash_attn`, `_FlashAttnP100`, `_expand_kv` and `reference`, with the P100
SIMT kernels replaced by tcgen05 tensor-core kernels in libfa_b200.so.

    from fa_p100 import flash_attn
    o = flash_attn(q, k, v, causal=True)   # q (B,Hq,N,D), k/v (B,Hkv,N,D), fp16 CUDA

D is 64 or 128, N is arbitrary, Hq a multiple of Hkv (MHA, GQA, MQA).
`full_precision` is accepted and ignored: the tensor cores multiply fp16
exactly and accumulate in fp32, which is the reference's fp32-MAC tier.
The backward follows the reference's flow: dq in fp32 (accumulated across key
blocks by TMA reduce-adds, so, like the reference's atomicAdd, not bitwise
deterministic), then cast to q's dtype. fa_p100_ext.backward_into with an fp16
dq takes the deterministic two-kernel backward instead.
"""
import math

import torch

import fa_p100_ext as _ext


class _FlashAttnP100(torch.autograd.Function):
    """fa_p100.py:31-45 of the reference."""

    @staticmethod
    def forward(ctx, q, k, v, causal, full_precision):
        o, lse = _ext.forward(q, k, v, causal, full_precision)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.causal = causal
        return o

    @staticmethod
    def backward(ctx, grad_o):
        q, k, v, o, lse = ctx.saved_tensors
        # dq comes back in fp32 and is cast to q's dtype (fa_p100.py:43-45)
        dq, dk, dv = _ext.backward(q, k, v, grad_o.contiguous(), o, lse, ctx.causal)
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), None, None


def flash_attn(q, k, v, causal=False, full_precision=False):
    """Attention over fp16 CUDA tensors (fa_p100.py:48-55).

    q is (B, Hq, N, D); k and v are (B, Hkv, N, D) with Hq a multiple of Hkv.
    Hkv == Hq is ordinary multi-head; Hkv == 1 is multi-query; anything between
    is grouped-query. N is arbitrary; D is 64 or 128.
    """
    return _FlashAttnP100.apply(q, k, v, causal, full_precision)


def _expand_kv(k, n_head):
    """K/V heads broadcast to `n_head` query heads; query head h reads kv head
    h // (n_head / Hkv) (the mapping of fa_p100.py:58-62)."""
    group = n_head // k.size(1)
    return k if group == 1 else torch.repeat_interleave(k, group, dim=1)


def reference(q, k, v, causal=False):
    """Plain-torch attention in fp32 for comparison, returned in q's dtype
    (the contract of fa_p100.py:65-75). Never used by flash_attn."""
    hq, n, d = q.size(1), q.size(2), q.size(3)
    kf = _expand_kv(k, hq).float()
    vf = _expand_kv(v, hq).float()
    logits = torch.einsum("bhid,bhjd->bhij", q.float(), kf) / math.sqrt(d)
    if causal:
        pos = torch.arange(n, device=q.device)
        logits = logits.masked_fill(pos[None, :] > pos[:, None], -math.inf)
    probs = torch.softmax(logits, dim=-1)
    return torch.einsum("bhij,bhjd->bhid", probs, vf).to(q.dtype)

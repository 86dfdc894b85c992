"""FlashAttention-2 for B200 (sm_100a) as a torch autograd Function.

Drop-in for the reference module of the same name (fa_p100.py): the same
`flash_attn`, `_FlashAttnP100`, `_expand_kv` and `reference`, with the P100
SIMT kernels replaced by tcgen05 tensor-core kernels in libfa_b200.so.

    from fa_p100 import flash_attn
    o = flash_attn(q, k, v, causal=True)   # q (B,Hq,N,D), k/v (B,Hkv,N,D), fp16 CUDA

D is 64 or 128, N is arbitrary, Hq a multiple of Hkv (MHA, GQA, MQA). The
tensors are fp16 (the reference's type) or, beyond it, bf16.
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
        dq, dk, dv = _grads(q, k, v, grad_o, o, lse, ctx.causal)
        return dq, dk, dv, None, None


def _grads(q, k, v, grad_o, o, lse, causal):
    """dq, dk, dv in the layouts of q, k, v (so autograd needs no copies to hand
    them on). dq is accumulated in fp32 and cast to q's dtype
    (fa_p100.py:43-45)."""
    dq32 = torch.empty_like(q, dtype=torch.float32)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    _ext.backward_into(q, k, v, grad_o, o, lse, causal, torch.float32, dq32, dk, dv)
    return dq32.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype)


class _FlashAttnBNHD(torch.autograd.Function):
    """flash_attn whose output is (B, N, Hq, D) contiguous: the layout an
    attention layer consumes next (the HF backend returns it transposed,
    fa_p100_hf.py:142). q, k, v are (B, H, N, D) views of any layout with a
    contiguous D axis, typically transposes of (B, N, H, D) projections; nothing
    is copied on the way in or out, and the gradients come back in the inputs'
    layouts."""

    @staticmethod
    def forward(ctx, q, k, v, causal, full_precision):
        B, H, N, D = q.shape
        out = torch.empty((B, N, H, D), device=q.device, dtype=q.dtype)
        o, lse = _ext.forward(q, k, v, causal, full_precision, o=out.transpose(1, 2))
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.causal = causal
        return out

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = _grads(q, k, v, grad_out.transpose(1, 2), o, lse, ctx.causal)
        return dq, dk, dv, None, None


def flash_attn_bnhd(q, k, v, causal=False, full_precision=False):
    """flash_attn with the output laid out (B, N, Hq, D) instead of (B, Hq, N, D)."""
    return _FlashAttnBNHD.apply(q, k, v, causal, full_precision)


def flash_attn(q, k, v, causal=False, full_precision=False):
    """Attention over fp16 (or bf16) CUDA tensors (fa_p100.py:48-55).

    q is (B, Hq, N, D); k and v are (B, Hkv, N, D) with Hq a multiple of Hkv.
    Hkv == Hq is ordinary multi-head; Hkv == 1 is multi-query; anything between
    is grouped-query. N is arbitrary; D is 64 or 128.
    """
    return _FlashAttnP100.apply(q, k, v, causal, full_precision)


def check_device_errors(device=None):
    """Synchronise `device` and raise RuntimeError if a kernel of this library
    gave up a bounded internal wait since the last check (its outputs are then
    incomplete). Each op also raises at the next call on its device once the
    asynchronous read of the error word it enqueued has landed."""
    _ext.check_device_errors(device)


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

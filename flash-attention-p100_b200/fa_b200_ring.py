"""Ring context-parallel attention across GPUs (long sequences).

The reference has no multi-GPU exchange at all (its multigpu.cu runs independent
forwards). This module splits one long causal sequence over G ranks, one
process per GPU, and passes K/V blocks around a ring with NCCL point-to-point
transfers over NVLink, so each GPU holds 1/G of the sequence and does 1/G of
the work.

Zigzag sharding: the sequence is cut into 2G chunks of C = N / (2G) rows; rank
r holds chunks r and 2G-1-r (concatenated, 2C rows), which gives every rank the
same amount of causal work. At ring step s rank r holds the K/V of rank
r' = (r - s) mod G and computes, with global positions:
  s = 0     local Q vs local K/V, causal over the 2C concatenated rows (the
            zigzag order makes the plain causal mask exact);
  r' < r    both local Q chunks vs remote chunk r' (entirely in the past),
            non-causal; remote chunk 2G-1-r' is entirely in the future;
  r' > r    local chunk 2G-1-r vs both remote chunks (both in the past),
            non-causal; local chunk r sees nothing.
Every piece is a C x C call of the single-GPU kernels. The forward merges the
pieces' (O, LSE) in fp32: LSE = logaddexp(a, b), O = O_a e^(a-LSE) + O_b e^(b-LSE).
The backward reruns the same pieces with the final O and LSE (so each piece's
Dv = rowsum(dO o O) and P = exp(S - LSE) are the global ones); dQ stays local
and the fp32 dK/dV accumulators travel around the ring with K/V, arriving back
at their owner after G hops. Transfers are double-buffered: the next step's
K/V are in flight while the current step computes.

The per-piece attention functions are injectable (`ops`), so the ring logic
runs on CPU ranks (gloo) in tests; the default ops are the CUDA kernels, which
also do the merge (one pass, fa_b200_merge_partial) and add each piece's
gradients straight into the fp32 dq and travelling dK/dV accumulators
(FA_B200_STAGE_ACCUMULATE), and read the pieces' Q/K/V/dO/O halves in place.
Ops without `merge` / `bwd_acc` get the plain torch versions below.
"""
import math
from contextlib import contextmanager

import torch
import torch.distributed as dist


@contextmanager
def _step_range(on_cuda, name):
    """An NVTX range named `name` around one ring step on CUDA tensors, so a
    profiler timeline (nsys, ncu's NVTX filters) shows each step's exchange and
    compute by name; nothing on CPU ranks."""
    if on_cuda:
        torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        if on_cuda:
            torch.cuda.nvtx.range_pop()


# ---------------------------------------------------------------------------
# zigzag layout
# ---------------------------------------------------------------------------
def zigzag_chunks(world, rank):
    """Global chunk ids (of 2*world) held by `rank`, in local order."""
    return rank, 2 * world - 1 - rank


def zigzag_shard(x, world, rank, dim=2):
    """The local 2C-row slice of a full tensor: chunks r and 2G-1-r along `dim`."""
    n = x.size(dim)
    if n % (2 * world):
        raise ValueError(f"sequence length {n} must be a multiple of 2 * world = {2 * world}")
    chunks = x.chunk(2 * world, dim=dim)
    a, b = zigzag_chunks(world, rank)
    return torch.cat([chunks[a], chunks[b]], dim=dim).contiguous()


def zigzag_unshard(parts, dim=2):
    """Inverse of zigzag_shard given every rank's local tensor (parts[r])."""
    world = len(parts)
    chunks = [None] * (2 * world)
    for r, t in enumerate(parts):
        a, b = zigzag_chunks(world, r)
        chunks[a], chunks[b] = t.chunk(2, dim=dim)
    return torch.cat(chunks, dim=dim)


def ring_pieces(world, rank, step):
    """The attention pieces of one ring step: a list of
    (q_half, kv_half, causal) with halves 0 = first local chunk, 1 = second,
    None = all 2C rows."""
    if step == 0:
        return [(None, None, True)]
    src = (rank - step) % world
    if src < rank:
        return [(0, 0, False), (1, 0, False)]
    return [(1, 0, False), (1, 1, False)]


def _half(t, h, dim=2):
    if h is None:
        return t
    c = t.size(dim) // 2
    return t.narrow(dim, h * c, c)


# ---------------------------------------------------------------------------
# local ops
# ---------------------------------------------------------------------------
class CudaOps:
    """The single-GPU kernels (fa_p100_ext): fp16 in, O fp16 + LSE fp32 out."""

    @staticmethod
    def fwd(q, k, v, causal):
        import fa_p100_ext
        return fa_p100_ext.forward(q, k, v, causal, False)

    @staticmethod
    def bwd(q, k, v, do, o, lse, causal):
        import fa_p100_ext
        dq, dk, dv = fa_p100_ext.backward(q, k, v, do, o, lse, causal)
        return dq, dk.float(), dv.float()

    @staticmethod
    def merge(o_acc, lse_acc, o_p, lse_p):
        import fa_p100_ext
        fa_p100_ext.merge_partial(o_acc, lse_acc, o_p, lse_p)

    @staticmethod
    def bwd_acc(q, k, v, do, o, lse, causal, dq, dk, dv):
        import fa_p100_ext
        fa_p100_ext.backward_accumulate(q, k, v, do, o, lse, causal, dq, dk, dv)


def _merge(o_acc, lse_acc, o_p, lse_p):
    """Fold one piece (O_p, LSE_p) into the running fp32 (O, LSE), in place."""
    lse_new = torch.logaddexp(lse_acc, lse_p)
    w_old = torch.exp(lse_acc - lse_new).unsqueeze(-1)
    w_new = torch.exp(lse_p - lse_new).unsqueeze(-1)
    o_acc.mul_(w_old).add_(o_p.float() * w_new)
    lse_acc.copy_(lse_new)


def _exchange(tensors, group, world, rank):
    """Send `tensors` to rank+1 and receive same-shaped ones from rank-1.
    Returns (received buffers, work handles to wait on)."""
    nxt, prv = (rank + 1) % world, (rank - 1) % world
    recv = [torch.empty_like(t) for t in tensors]
    ops = []
    for t, r in zip(tensors, recv):
        ops.append(dist.P2POp(dist.isend, t, nxt, group))
        ops.append(dist.P2POp(dist.irecv, r, prv, group))
    works = dist.batch_isend_irecv(ops)
    return recv, works


def ring_forward(q, k, v, ops=CudaOps, group=None):
    """Causal ring attention on zigzag shards. q (B,Hq,2C,D), k/v (B,Hkv,2C,D)
    local. Returns (O fp16-castable fp32 accumulator, LSE fp32)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    o_acc = None
    lse_acc = None
    kv = (k.contiguous(), v.contiguous())
    for step in range(world):
        with _step_range(q.is_cuda, f"ring fwd step {step}/{world}"):
            nxt = None
            if step + 1 < world:
                nxt = _exchange(kv, group, world, rank)
            merge = getattr(ops, "merge", _merge)
            for qh, kh, causal in ring_pieces(world, rank, step):
                o_p, lse_p = ops.fwd(_half(q, qh), _half(kv[0], kh), _half(kv[1], kh), causal)
                if o_acc is None:
                    o_acc, lse_acc = o_p.float(), lse_p.float().clone()
                    continue
                merge(_half(o_acc, qh), _half(lse_acc, qh), o_p, lse_p)
            if nxt is not None:
                bufs, works = nxt
                for w in works:
                    w.wait()
                kv = tuple(bufs)
    return o_acc, lse_acc


def ring_backward(q, k, v, do, o, lse, ops=CudaOps, group=None):
    """Gradients of ring_forward. o, lse: the final local O and LSE. Returns
    dq (fp32), dk, dv (fp32) for the local shards."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    dq = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
    kv = (k.contiguous(), v.contiguous())
    acc = None           # (dK, dV) accumulators of the K/V block currently held
    acc_in = None        # accumulators in flight toward this rank
    for step in range(world):
        with _step_range(q.is_cuda, f"ring bwd step {step}/{world}"):
            nxt = None
            if step + 1 < world:
                nxt = _exchange(kv, group, world, rank)
            dk_s = torch.zeros(kv[0].shape, dtype=torch.float32, device=q.device)
            dv_s = torch.zeros_like(dk_s)
            for qh, kh, causal in ring_pieces(world, rank, step):
                args = (_half(q, qh), _half(kv[0], kh), _half(kv[1], kh), _half(do, qh),
                        _half(o, qh), _half(lse, qh), causal)
                if hasattr(ops, "bwd_acc"):
                    ops.bwd_acc(*args, _half(dq, qh), _half(dk_s, kh), _half(dv_s, kh))
                    continue
                dq_p, dk_p, dv_p = ops.bwd(*args)
                _half(dq, qh).add_(dq_p)
                _half(dk_s, kh).add_(dk_p)
                _half(dv_s, kh).add_(dv_p)
            # this block's accumulators arrive from the previous rank (none at step 0)
            if acc_in is not None:
                bufs, works = acc_in
                for w in works:
                    w.wait()
                dk_s.add_(bufs[0])
                dv_s.add_(bufs[1])
            acc = (dk_s, dv_s)
            # pass the accumulators on with the K/V block; after the last step this
            # hop brings them home to their owner
            acc_in = _exchange(acc, group, world, rank)
            if nxt is not None:
                bufs, works = nxt
                for w in works:
                    w.wait()
                kv = tuple(bufs)
    bufs, works = acc_in
    for w in works:
        w.wait()
    return dq, bufs[0], bufs[1]


class _RingAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, group, ops):
        o_acc, lse = ring_forward(q, k, v, ops, group)
        o = o_acc.to(q.dtype)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.group, ctx.ops = group, ops
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = ring_backward(q, k, v, do.contiguous(), o, lse, ctx.ops, ctx.group)
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), None, None


def ring_flash_attn(q, k, v, group=None, ops=CudaOps):
    """Causal attention of one long sequence sharded zigzag across the ranks of
    `group`: q (B,Hq,2C,D), k/v (B,Hkv,2C,D) are this rank's zigzag_shard of
    the full tensors; returns this rank's shard of O. Differentiable."""
    if q.size(2) % 2:
        raise ValueError("local shard length must be even (two chunks)")
    return _RingAttention.apply(q, k, v, group, ops)


def ring_flops(B, Hq, N, D):
    """Algorithmic causal fwd+bwd FLOPs of the whole (unsharded) problem."""
    return 3.5 * 4.0 * B * Hq * D * N * (N + 1) / 2

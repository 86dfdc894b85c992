"""Ring context parallelism on CPU ranks (gloo), with the oracle as the
per-piece attention: the zigzag pairing, the LSE merge, the K/V rotation and
the travelling dK/dV accumulators are checked against single-process attention
over the whole sequence. No GPU involved."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import fa_b200_ring as ring


class OracleOps:
    """Per-piece attention on the CPU oracle (fp32)."""

    @staticmethod
    def fwd(q, k, v, causal):
        from oracle import attention_oracle as orc
        return orc.attention(q, k, v, causal, with_lse=True)

    @staticmethod
    def bwd(q, k, v, do, o, lse, causal):
        from oracle import attention_oracle as orc
        return orc.attention_grads_given_lse(q, k, v, do, o, lse, causal)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_ring_pieces_cover_every_causal_pair_once(world):
    """Over all ring steps, each local query chunk meets each earlier-or-equal
    key chunk exactly once, and never a later one."""
    for rank in range(world):
        local = ring.zigzag_chunks(world, rank)
        seen = {}
        for step in range(world):
            src = (rank - step) % world
            remote = ring.zigzag_chunks(world, src)
            for qh, kh, causal in ring.ring_pieces(world, rank, step):
                qs = local if qh is None else (local[qh],)
                ks = remote if kh is None else (remote[kh],)
                for qc in qs:
                    for kc in ks:
                        if causal and kc > qc:
                            continue          # masked out by the causal piece
                        seen[(qc, kc)] = seen.get((qc, kc), 0) + 1
        want = {(qc, kc): 1 for qc in local for kc in range(2 * world) if kc <= qc}
        assert seen == want


def test_zigzag_roundtrip():
    x = torch.arange(2 * 3 * 24 * 4, dtype=torch.float32).reshape(2, 3, 24, 4)
    parts = [ring.zigzag_shard(x, 3, r) for r in range(3)]
    assert torch.equal(ring.zigzag_unshard(parts), x)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, shape, seed, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from oracle import attention_oracle as orc
        B, Hq, Hkv, N, D = shape
        q, k, v, do = (t.float() for t in orc.seeded_inputs(B, Hq, Hkv, N, D, seed=seed))
        loc = [ring.zigzag_shard(t, world, rank).requires_grad_(i < 3)
               for i, t in enumerate((q, k, v, do))]
        o = ring.ring_flash_attn(loc[0], loc[1], loc[2], ops=OracleOps)
        o.backward(loc[3])
        out[rank] = [o.detach(), loc[0].grad, loc[1].grad, loc[2].grad]
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,shape", [(2, (1, 4, 2, 32, 64)), (3, (2, 2, 1, 36, 64))])
def test_ring_matches_full_sequence(world, shape):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(world, _free_port(), shape, 3, out), nprocs=world,
                           join=True, start_method="spawn")
        res = [out[r] for r in range(world)]
    from oracle import attention_oracle as orc
    B, Hq, Hkv, N, D = shape
    q, k, v, do = orc.seeded_inputs(B, Hq, Hkv, N, D, seed=3)
    ro = orc.attention(q, k, v, True)
    rq, rk, rv = orc.attention_grads(q, k, v, do, True)
    for i, ref in enumerate((ro, rq, rk, rv)):
        got = ring.zigzag_unshard([res[r][i] for r in range(world)])
        assert (got - ref).abs().max().item() < 1e-4, i


def _dead_rank_worker(rank, world, port, out):
    """Rank 1 leaves before the ring starts; rank 0 must fail within the
    process-group timeout instead of hanging."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    import time
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        return   # exits without joining the ring
    q = torch.zeros(1, 1, 8, 64)
    t0 = time.time()
    try:
        ring.ring_forward(q, q, q, ops=OracleOps)
        out[rank] = "no error"
    except Exception as e:  # the peer is gone: gloo raises
        out[rank] = f"raised after {time.time() - t0:.1f}s: {type(e).__name__}"


def test_ring_peer_failure_raises():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_dead_rank_worker, args=(2, _free_port(), out), nprocs=2, join=True,
                           start_method="spawn")
        assert out[0].startswith("raised"), out[0]

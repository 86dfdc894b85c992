"""Parity of the sm_100a kernels with the CPU oracle, through the reference's
own API (flash_attn / the autograd Function), on the reference's test matrix
(test_fa_p100.py:56-139): both head dims, MHA/GQA/MQA, sequence lengths that
straddle every tile edge, causal and not, and the four input regimes.

Gate: the reference's metric rel = max|got-ref|/rms(ref) < 6e-2
(test_fa_p100.py:24, :35-37) on O and on dQ/dK/dV, plus the tighter
Frobenius relative error < 1e-2 on the gradients and an LSE check.
"""
import pytest
import torch

from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu

TOL = 6e-2          # reference's regression tolerance on `rel`
GRAD_FROB = 1e-2    # north-star gradient tolerance (Frobenius relative)
LSE_ABS = 2e-3      # |LSE - oracle| in natural-log units


def _nan(shape, dtype, dev):
    """An output buffer filled with NaN before the launch, so a tile the kernel
    never writes cannot pass by inheriting earlier correct bytes."""
    return torch.full(shape, float("nan"), dtype=dtype, device=dev)


def _run_fwd(q, k, v, causal, dev):
    import fa_p100_ext
    B, H, N, _ = q.shape
    o, lse = fa_p100_ext.forward(q.to(dev), k.to(dev), v.to(dev), causal, False,
                                 o=_nan(q.shape, q.dtype, dev), lse=_nan((B, H, N), torch.float32, dev))
    torch.cuda.synchronize()
    import _lib
    assert _lib.device_error(0) == 0
    return o.cpu(), lse.cpu()


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("Hq,Hkv", [(8, 8), (8, 2), (8, 1)])
@pytest.mark.parametrize("N", [1, 7, 63, 64, 65, 333, 1023])
@pytest.mark.parametrize("causal", [False, True])
def test_forward(cuda, D, Hq, Hkv, N, causal):
    q, k, v, _ = orc.seeded_inputs(1, Hq, Hkv, N, D, seed=N * 7 + D + Hkv)
    o, lse = _run_fwd(q, k, v, causal, cuda)
    ro, rlse = orc.attention(q, k, v, causal, with_lse=True)
    assert torch.isfinite(o.float()).all() and torch.isfinite(lse).all()
    e = orc.rel(o, ro)
    assert e < TOL, f"rel {e:.3e}"
    assert (lse - rlse).abs().max().item() < LSE_ABS


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("Hq,Hkv", [(4, 4), (8, 2), (8, 1)])
@pytest.mark.parametrize("N", [7, 64, 129, 333])
@pytest.mark.parametrize("causal", [False, True])
def test_gradients(cuda, D, Hq, Hkv, N, causal):
    import fa_p100
    q, k, v, do = orc.seeded_inputs(1, Hq, Hkv, N, D, seed=1000 + N + D + Hkv)
    a = [t.to(cuda).requires_grad_(True) for t in (q, k, v)]
    fa_p100.flash_attn(*a, causal, True).backward(do.to(cuda))
    torch.cuda.synchronize()
    rq, rk, rv = orc.attention_grads(q, k, v, do, causal)
    for name, got, ref in zip("QKV", (a[0].grad, a[1].grad, a[2].grad), (rq, rk, rv)):
        assert got.dtype == torch.float16
        r = orc.rel(got, ref)
        f = orc.frob_rel(got, ref)
        assert r < TOL and f < GRAD_FROB, f"d{name}: rel {r:.3e} frob {f:.3e}"
    # the same gradients into NaN-filled outputs, through both backward paths
    # (fused with fp32 dq, and the deterministic dK/dV + dQ kernels with fp16 dq)
    import fa_p100_ext
    qd, kd, vd, dod = (t.to(cuda) for t in (q, k, v, do))
    o, lse = fa_p100_ext.forward(qd, kd, vd, causal)
    for dq_dtype in (torch.float32, torch.float16):
        dq, dk, dv = fa_p100_ext.backward_into(
            qd, kd, vd, dod, o, lse, causal, dq_dtype, dq=_nan(qd.shape, dq_dtype, cuda),
            dk=_nan(kd.shape, kd.dtype, cuda), dv=_nan(vd.shape, vd.dtype, cuda))
        torch.cuda.synchronize()
        for name, got, ref in zip("QKV", (dq, dk, dv), (rq, rk, rv)):
            assert torch.isfinite(got.float()).all(), f"d{name} ({dq_dtype} dq): unwritten entries"
            f = orc.frob_rel(got, ref)
            assert f < GRAD_FROB, f"d{name} ({dq_dtype} dq): frob {f:.3e}"


@pytest.mark.parametrize("regime", [1.0, 10.0, 0.05, 3.0])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
def test_input_regimes(cuda, regime, D, causal):
    """test_fa_p100.py:107-139: q and k scaled by x1, x10, x0.05, x3; v, dO N(0,1)."""
    import fa_p100
    q, k, v, do = orc.seeded_inputs(1, 4, 4, 256, D, seed=77, qk_scale=regime)
    a = [t.to(cuda).requires_grad_(True) for t in (q, k, v)]
    o = fa_p100.flash_attn(*a, causal, True)
    o.backward(do.to(cuda))
    torch.cuda.synchronize()
    ro = orc.attention(q, k, v, causal)
    assert orc.rel(o.detach(), ro) < TOL
    rq, rk, rv = orc.attention_grads(q, k, v, do, causal)
    for got, ref in zip((a[0].grad, a[1].grad, a[2].grad), (rq, rk, rv)):
        assert orc.rel(got, ref) < TOL


@pytest.mark.parametrize("D,causal", [(64, True), (128, False)])
def test_backward_op_contract(cuda, D, causal):
    """fa_p100_ext.backward returns dq fp32 (B,Hq,N,D) and dk/dv fp16 (B,Hkv,N,D),
    like fa_p100_ext.cu:121-123 (fused kernel, atomic dQ); the fp16-dq path (separate
    kernels) agrees with it and is bitwise deterministic."""
    import fa_p100_ext
    q, k, v, do = orc.seeded_inputs(2, 4, 2, 200, D, seed=5)
    q, k, v, do = (t.to(cuda) for t in (q, k, v, do))
    o, lse = fa_p100_ext.forward(q, k, v, causal, False)
    dq, dk, dv = fa_p100_ext.backward(q, k, v, do, o, lse, causal)
    assert dq.dtype == torch.float32 and dq.shape == q.shape
    assert dk.dtype == torch.float16 and dk.shape == k.shape and dv.shape == v.shape
    dq16, dk2, dv2 = fa_p100_ext.backward_into(q, k, v, do, o, lse, causal, torch.float16)
    dq16b, dk3, dv3 = fa_p100_ext.backward_into(q, k, v, do, o, lse, causal, torch.float16)
    assert torch.equal(dq16, dq16b) and torch.equal(dk2, dk3) and torch.equal(dv2, dv3)
    for a, b in ((dq, dq16), (dk, dk2), (dv, dv2)):
        assert orc.frob_rel(a, b) < 2e-3
    rq, rk, rv = orc.attention_grads(q, k, v, do, causal)
    for got, ref in ((dq, rq), (dk, rk), (dv, rv), (dq16, rq)):
        assert orc.frob_rel(got, ref) < 1e-2


@pytest.mark.parametrize("D,causal,Hq,Hkv,N", [(64, True, 4, 2, 333), (128, False, 8, 1, 700),
                                               (128, True, 4, 4, 1024)])
def test_fused_stage_matches(cuda, D, causal, Hq, Hkv, N):
    """The fused stage requested explicitly (rows-only workspace, so no group
    split) against the oracle and against the extension op."""
    import _lib
    import fa_p100_ext
    q, k, v, do = (t.to(cuda) for t in orc.seeded_inputs(1, Hq, Hkv, N, D, seed=8))
    o, lse = fa_p100_ext.forward(q, k, v, causal, False)
    lib = _lib.lib()
    dq = _nan(q.shape, torch.float32, cuda)
    dk, dv = _nan(k.shape, k.dtype, cuda), _nan(v.shape, v.dtype, cuda)
    ws_b = lib.fa_b200_backward_workspace_bytes(1, Hq, N)
    ws = torch.empty(ws_b // 4, device=cuda)
    st = lib.fa_b200_backward_stages(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(),
                                     o.data_ptr(), lse.data_ptr(), dq.data_ptr(), 1, dk.data_ptr(),
                                     dv.data_ptr(), ws.data_ptr(), ws_b, 1, Hq, Hkv, N, D,
                                     int(causal), 1 | 8, torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "fused stage")
    torch.cuda.synchronize()
    assert _lib.device_error(0) == 0
    rq, rk, rv = orc.attention_grads(q, k, v, do, causal)
    for got, ref in ((dq, rq), (dk, rk), (dv, rv)):
        assert orc.frob_rel(got, ref) < 1e-2
    dq2, dk2, dv2 = fa_p100_ext.backward(q, k, v, do, o, lse, causal)
    if Hq == Hkv:   # nothing to split: the same kernel, the same dK/dV bits
        assert torch.equal(dk, dk2) and torch.equal(dv, dv2)
    else:           # the op's workspace lets small GQA grids split (fp32 partial sums)
        assert orc.frob_rel(dk, dk2) < 1e-3 and orc.frob_rel(dv, dv2) < 1e-3
    assert orc.frob_rel(dq, dq2) < 1e-4


@pytest.mark.parametrize("B,Hq,Hkv,N,D", [(2, 16, 1, 1537, 64), (1, 8, 2, 700, 128), (3, 6, 3, 260, 128)])
def test_gqa_group_split_matches_unsplit(cuda, B, Hq, Hkv, N, D):
    """With the larger workspace the fused backward splits small GQA/MQA grids
    over several CTAs and adds partial dK/dV in fp32; with the rows-only
    workspace it does not. Both must give the same gradients up to the order of
    fp32 additions."""
    import _lib
    import fa_p100_ext
    g = torch.Generator(device="cuda").manual_seed(11)
    mk = lambda h: torch.randn(B, h, N, D, device="cuda", generator=g).half()
    q, k, v, do = mk(Hq), mk(Hkv), mk(Hkv), mk(Hq)
    o, lse = fa_p100_ext.forward(q, k, v, True)
    split = fa_p100_ext.backward(q, k, v, do, o, lse, True)           # gqa-sized workspace
    lib = _lib.lib()
    dq = _nan(q.shape, torch.float32, cuda)
    dk, dv = _nan(k.shape, k.dtype, cuda), _nan(v.shape, v.dtype, cuda)
    ws_bytes = lib.fa_b200_backward_workspace_bytes(B, Hq, N)          # rows only: no split
    ws = torch.empty(ws_bytes // 4, device="cuda")
    st = lib.fa_b200_backward(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(),
                              o.data_ptr(), lse.data_ptr(), dq.data_ptr(), 1, dk.data_ptr(),
                              dv.data_ptr(), ws.data_ptr(), ws_bytes, B, Hq, Hkv, N, D, 1,
                              torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "fa_b200_backward")
    for a, b in zip(split, (dq, dk, dv)):
        a, b = a.float(), b.float()
        assert (a - b).norm().item() <= 2e-3 * b.norm().item()
    assert _lib.device_error(0) == 0


@pytest.mark.parametrize("N,D,causal", [(1024, 128, True), (1000, 64, True), (777, 128, False),
                                         (2048, 64, False)])
def test_small_grid_forward_matches_two_tile(cuda, N, D, causal):
    """The forward launches one of two kernels by grid size: the two-tile one
    (256 query rows per CTA) when B*Hq*ceil(N/256) fills the GPU, the
    small-grid one (128 rows per CTA, 256-key steps) otherwise. The same heads
    computed inside a large batch of heads and on their own take the two
    paths; O and LSE must agree to rounding and both meet the oracle."""
    import _lib
    import fa_p100_ext
    g = torch.Generator(device="cuda").manual_seed(21)
    H = 160                                   # 160 * ceil(N/256) >= 148: two-tile kernel
    mk = lambda h: torch.randn(1, h, N, D, device="cuda", generator=g).half()
    q, k, v = mk(H), mk(H), mk(H)
    o_big, lse_big = fa_p100_ext.forward(q, k, v, causal)
    qs, ks, vs = (t[:, :4].contiguous() for t in (q, k, v))   # 4 heads: small-grid kernel
    o_small, lse_small = fa_p100_ext.forward(qs, ks, vs, causal)
    assert (o_small.float() - o_big[:, :4].float()).abs().max().item() <= 2e-3
    assert (lse_small - lse_big[:, :4]).abs().max().item() <= 1e-4
    rq = orc.attention(qs, ks, vs, causal, device=cuda)
    assert orc.rel(o_small, rq) < 6e-2
    assert _lib.device_error(0) == 0


@pytest.mark.parametrize("H", [4, 160])            # small-grid and two-tile forward
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_causal_first_row_is_v0(cuda, H, D, dtype):
    """A causal row 0 sees key 0 alone: its weight is exp(0) = 1 whatever the
    score, so O[row 0] is V[0] to the last bit. This holds only if the row
    maximum the softmax subtracts is exactly the row's largest score (P's
    16-bit rounding then agrees with the fp32 row sum), so it pins the max
    reduction over the masked S row."""
    import fa_p100_ext
    g = torch.Generator(device="cuda").manual_seed(3)
    mk = lambda: (3 * torch.randn(1, H, 1024, D, device="cuda", generator=g)).to(dtype)
    q, k, v = mk(), mk(), mk()
    o, _ = fa_p100_ext.forward(q, k, v, True)
    assert torch.equal(o[:, :, 0], v[:, :, 0])

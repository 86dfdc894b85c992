"""Strided layouts through the same kernels: q, k, v, dO, o as (B, H, N, D)
views of (B, N, H, D) storage (what attention layers produce), and of rows
padded inside a wider buffer, must give exactly the contiguous results -- the
forward and the deterministic backward bit for bit, the fused backward (whose
fp32 adds are unordered) to fp32 rounding. The layout-preserving autograd path used
by the HF backend is checked against flash_attn."""
import pytest
import torch

import fa_p100
import fa_p100_ext

pytestmark = pytest.mark.gpu

CASES = [  # B, Hq, Hkv, N, D, causal
    # B*Hq*ceil(N/256) below the SM count: the small-grid forward
    (2, 4, 2, 300, 64, True),
    (1, 8, 8, 1000, 128, False),
    (2, 6, 1, 513, 128, True),
    # enough 256-row blocks to fill the GPU: the two-tile forward
    (2, 40, 8, 1000, 128, True),
    (1, 80, 80, 600, 64, False),
]


def bnhd(t):
    """The same values as t (B, H, N, D), stored (B, N, H, D)."""
    return t.transpose(1, 2).contiguous().transpose(1, 2)


def padded(t):
    """The same values as t, each row stored in a row of 2D elements."""
    B, H, N, D = t.shape
    buf = torch.zeros(B, H, N, 2 * D, device=t.device, dtype=t.dtype)
    buf[..., :D] = t
    return buf[..., :D]


def inputs(B, Hq, Hkv, N, D, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda h: torch.randn(B, h, N, D, device="cuda", generator=g).half()
    return mk(Hq), mk(Hkv), mk(Hkv), mk(Hq)


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(map(str, c)))
@pytest.mark.parametrize("layout", [bnhd, padded], ids=["bnhd", "padded"])
def test_strided_matches_contiguous(cuda, case, layout):
    B, Hq, Hkv, N, D, causal = case
    q, k, v, do = inputs(B, Hq, Hkv, N, D)
    o, lse = fa_p100_ext.forward(q, k, v, causal)
    qs, ks, vs, dos = (layout(t) for t in (q, k, v, do))
    assert not qs.is_contiguous()
    o2, lse2 = fa_p100_ext.forward(qs, ks, vs, causal)
    assert torch.equal(o, o2) and torch.equal(lse, lse2)
    # output written into a strided buffer
    o3, _ = fa_p100_ext.forward(qs, ks, vs, causal, o=layout(torch.full_like(q, float('nan'))))
    assert torch.equal(o, o3)
    os_ = layout(o)
    # deterministic backward (fp16 dq): every gradient bit for bit
    ref16 = fa_p100_ext.backward_into(q, k, v, do, o, lse, causal, torch.float16)
    got16 = fa_p100_ext.backward_into(qs, ks, vs, dos, os_, lse, causal, torch.float16,
                                      layout(torch.full_like(q, float('nan'))), layout(torch.full_like(k, float('nan'))),
                                      layout(torch.full_like(v, float('nan'))))
    for a, b in zip(ref16, got16):
        assert torch.equal(a, b)
    # fused backward (fp32 dq): dQ -- and dK/dV where a small GQA grid splits
    # its group over CTAs that add fp32 partials -- to the order of fp32 adds
    ref = fa_p100_ext.backward(q, k, v, do, o, lse, causal)
    got = fa_p100_ext.backward_into(qs, ks, vs, dos, os_, lse, causal, torch.float32,
                                    layout(torch.full(q.shape, float("nan"), device="cuda")),
                                    layout(torch.full_like(k, float('nan'))), layout(torch.full_like(v, float('nan'))))
    for a, b in zip(ref, got):
        a, b = a.float(), b.float()
        assert (a - b).norm().item() <= 1e-3 * a.norm().item()


def test_bnhd_autograd_matches_flash_attn(cuda):
    """The HF backend's path: projections stored (B, N, H, D), output straight
    in (B, N, H, D), gradients in the inputs' layouts."""
    B, Hq, Hkv, N, D = 1, 16, 8, 700, 128
    q, k, v, do = inputs(B, Hq, Hkv, N, D, seed=3)
    leaves = [t.transpose(1, 2).contiguous().requires_grad_(True) for t in (q, k, v)]
    out = fa_p100.flash_attn_bnhd(*(t.transpose(1, 2) for t in leaves), True)
    assert out.shape == (B, N, Hq, D) and out.is_contiguous()
    out.backward(do.transpose(1, 2))
    ref_in = [t.clone().requires_grad_(True) for t in (q, k, v)]
    ref = fa_p100.flash_attn(*ref_in, True)
    ref.backward(do)
    assert torch.equal(out.transpose(1, 2), ref)
    for leaf, r in zip(leaves, ref_in):
        assert leaf.grad.is_contiguous()     # (B, N, H, D) like the projection
        g, rg = leaf.grad.transpose(1, 2).float(), r.grad.float()
        assert (g - rg).norm().item() <= 1e-3 * rg.norm().item()

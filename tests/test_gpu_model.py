"""Model-level parity through the HF registration (the method of the
reference's verify_hf.py:78-96, :131-160, on a small random-init Qwen3 since no
weights are available here): the deviation of fa_p100's logits from sdpa's must
stay within 2x (mean) and 4x (p99.99) of the eager-vs-sdpa deviation, the loss
gap under 1e-3 nats, and a training step must produce finite gradients."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _model(impl, dev):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    cfg = Qwen3Config(vocab_size=2048, hidden_size=256, intermediate_size=768,
                      num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=64, max_position_embeddings=4096, initializer_range=0.02,
                      rope_parameters={"rope_theta": 1e6, "rope_type": "default"},
                      tie_word_embeddings=True, attn_implementation="sdpa" if impl == "fa_p100" else impl)
    torch.manual_seed(0)
    with torch.device(dev):
        m = Qwen3ForCausalLM(cfg)
    if impl == "fa_p100":
        import fa_p100_hf
        fa_p100_hf.enable_fa_p100(m)
    return m.eval()


def test_qwen3_logits_envelope(cuda):
    ids = torch.randint(0, 2048, (2, 1000), generator=torch.Generator().manual_seed(1)).to(cuda)
    out = {}
    for impl in ("sdpa", "eager", "fa_p100"):
        m = _model(impl, cuda)
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.float16):
            r = m(input_ids=ids, labels=ids)
        out[impl] = (r.logits.float(), r.loss.item())
    ref = out["sdpa"][0]
    dev_eager = (out["eager"][0] - ref).abs().flatten()
    dev_fa = (out["fa_p100"][0] - ref).abs().flatten()
    m_e, m_f = dev_eager.mean().item(), dev_fa.mean().item()
    q = lambda t: torch.quantile(t[::max(1, t.numel() // 1_000_000)], 0.9999).item()
    print(f"mean dev: fa {m_f:.3e} eager {m_e:.3e}; loss fa {out['fa_p100'][1]:.5f} "
          f"sdpa {out['sdpa'][1]:.5f}")
    assert m_f <= 2 * m_e + 1e-6
    assert q(dev_fa) <= 4 * q(dev_eager) + 1e-5
    assert abs(out["fa_p100"][1] - out["sdpa"][1]) < 1e-3


def test_qwen3_training_step_gradients(cuda):
    m = _model("fa_p100", cuda).train()
    ids = torch.randint(0, 2048, (1, 777), generator=torch.Generator().manual_seed(2)).to(cuda)
    with torch.autocast("cuda", dtype=torch.float16):
        loss = m(input_ids=ids, labels=ids).loss
    loss.backward()
    grads = [p.grad for p in m.parameters() if p.grad is not None]
    assert len(grads) > 10 and all(torch.isfinite(g).all() for g in grads)


def test_hf_output_dtype_follows_autocast(cuda):
    """Qwen3-style inputs (q, k fp32 after their fp32 norm weights, v fp16):
    under autocast the backend's output keeps the autocast dtype, as SDPA's
    does; outside autocast it returns in q's dtype. The values agree exactly."""
    import warnings
    import fa_p100_hf

    class _Layer:
        is_causal = True

    g = torch.Generator(device=cuda).manual_seed(5)
    q = torch.randn(1, 4, 200, 64, device=cuda, generator=g)
    k = torch.randn(1, 2, 200, 64, device=cuda, generator=g)
    v = torch.randn(1, 2, 200, 64, device=cuda, generator=g).half()
    with torch.autocast("cuda", dtype=torch.float16):
        o16, _ = fa_p100_hf.fa_p100_attention_forward(_Layer(), q, k, v, None)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        ob16, _ = fa_p100_hf.fa_p100_attention_forward(_Layer(), q, k, v.bfloat16(), None)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        o32, _ = fa_p100_hf.fa_p100_attention_forward(_Layer(), q, k, v, None)
    assert o16.dtype == torch.float16 and ob16.dtype == torch.bfloat16 and o32.dtype == torch.float32
    assert o16.shape == (1, 200, 4, 64)
    assert torch.equal(o16.float(), o32)
    ref = torch.nn.functional.scaled_dot_product_attention(
        q.half(), k.half().repeat_interleave(2, 1), v.repeat_interleave(2, 1), is_causal=True)
    assert (ob16.float() - ref.transpose(1, 2).float()).abs().max().item() < 5e-2

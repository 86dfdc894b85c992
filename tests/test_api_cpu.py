"""The Python boundary without a GPU: the reference's op validation
(fa_p100_ext.cu:31-35, :55-65) and every HF guard (fa_p100_hf.py:64-105,
:183-211) fire before any kernel is reached."""
import math

import pytest
import torch

import fa_p100
import fa_p100_ext
import fa_p100_hf


def t(*shape, dtype=torch.float16):
    return torch.zeros(*shape, dtype=dtype)


def test_ops_reject_cpu_tensors_like_the_reference():
    with pytest.raises(RuntimeError, match="q must be a CUDA tensor"):
        fa_p100_ext.forward(t(1, 2, 8, 64), t(1, 2, 8, 64), t(1, 2, 8, 64), False, False)
    with pytest.raises(RuntimeError, match="q must be a CUDA tensor"):
        fa_p100_ext.backward(*(t(1, 2, 8, 64) for _ in range(5)), t(1, 2, 8, dtype=torch.float32),
                             True)
    with pytest.raises(RuntimeError, match="q must be a CUDA tensor"):
        fa_p100.flash_attn(t(1, 2, 8, 64), t(1, 2, 8, 64), t(1, 2, 8, 64))


def test_reference_function_matches_oracle_formula():
    """fa_p100.reference keeps the reference's contract (fp32 math, input dtype out)."""
    from oracle import attention_oracle as orc
    q, k, v, _ = orc.seeded_inputs(1, 4, 2, 19, 64, seed=3)
    for causal in (False, True):
        got = fa_p100.reference(q.float(), k.float(), v.float(), causal)
        want = orc.attention(q, k, v, causal)
        assert (got - want).abs().max().item() < 1e-5
        assert fa_p100.reference(q, k, v, causal).dtype == torch.float16


class _Mod:
    is_causal = True


def hf(q=None, k=None, mask=None, dropout=0.0, scaling=None, **kw):
    q = t(1, 4, 8, 64) if q is None else q
    k = t(1, 2, 8, 64) if k is None else k
    return fa_p100_hf.fa_p100_attention_forward(_Mod(), q, k, k, mask, dropout, scaling, None,
                                                **kw)


@pytest.mark.parametrize("kwargs,match", [
    (dict(mask=t(1, 1, 8, 8)), "attention mask"),
    (dict(output_attentions=True), "output_attentions"),
    (dict(head_mask=t(4)), "head_mask"),
    (dict(sliding_window=128), "sliding window"),
    (dict(dropout=0.1), "dropout"),
    (dict(q=t(1, 4, 8, 96), k=t(1, 2, 8, 96)), "head_dim"),
    (dict(scaling=0.2), "1/sqrt"),
    (dict(k=t(1, 2, 9, 64)), "equal query and key lengths"),
])
def test_hf_guards_raise(kwargs, match):
    with pytest.raises(NotImplementedError, match=match):
        hf(**kwargs)


def test_hf_scaling_equal_to_default_is_accepted_until_the_kernel():
    # the guard passes, then the op rejects the CPU tensor (no silent fallback)
    with pytest.raises(RuntimeError, match="CUDA"):
        hf(scaling=1 / math.sqrt(64))


def _tiny_qwen3():
    from transformers import Qwen3Config, Qwen3ForCausalLM
    cfg = Qwen3Config(vocab_size=64, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=2, num_key_value_heads=1, head_dim=64,
                      max_position_embeddings=64, tie_word_embeddings=True)
    return Qwen3ForCausalLM(cfg)


def test_register_and_enable():
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    assert fa_p100_hf.register() == "fa_p100"
    assert ALL_ATTENTION_FUNCTIONS["fa_p100"] is fa_p100_hf.fa_p100_attention_forward
    model = fa_p100_hf.enable_fa_p100(_tiny_qwen3(), full_precision=True)
    assert model.config._attn_implementation == "fa_p100"
    assert model.config.use_cache is False
    assert all(getattr(m, "_fa_p100_full_precision", None) is True for m in model.modules())
    ids = torch.zeros(1, 8, dtype=torch.long)
    with pytest.raises(NotImplementedError, match="padding mask"):
        model(ids, attention_mask=torch.tensor([[1, 1, 1, 1, 1, 1, 0, 0]]))
    with pytest.raises(NotImplementedError, match="KV cache"):
        model(ids, use_cache=True)
    # idempotent: enabling twice keeps a single guard
    assert fa_p100_hf.enable_fa_p100(model) is model


def test_finetune_harness_host_parts():
    """The harness's data and model description, without a GPU: synthetic
    blocks are reproducible, the default model is Qwen3-0.6B's architecture,
    and the CLI defaults follow the reference's (seq 2048, 30 steps, 3 warm-up,
    8 blocks, 8 loss chunks)."""
    import finetune_hf
    a = finetune_hf.synthetic_blocks(1000, 64, 3, seed=4)
    b = finetune_hf.synthetic_blocks(1000, 64, 3, seed=4)
    assert a.shape == (3, 64) and (a == b).all() and a.max() < 1000
    cfg = finetune_hf.qwen3_0p6b_config()
    assert (cfg.num_hidden_layers, cfg.hidden_size, cfg.num_attention_heads,
            cfg.num_key_value_heads, cfg.head_dim, cfg.vocab_size) == (28, 1024, 16, 8, 128, 151936)
    args = finetune_hf.parser().parse_args([])
    assert (args.seq_len, args.steps, args.warmup, args.blocks, args.loss_chunks) == (2048, 30, 3, 8, 8)

"""HuggingFace transformers attention backend named "fa_p100", backed by the
B200 kernels. Same public surface as the reference module (fa_p100_hf.py):

    from fa_p100_hf import enable_fa_p100
    enable_fa_p100(model)                 # model runs attention through flash_attn

Contract kept from the reference (fa_p100_hf.py:46-213):
  * inputs arrive (B, H, N, D) with K/V un-expanded (GQA/MQA handled by the
    kernel), the output goes back (B, N, H, D) plus None for the weights;
  * no attention-mask function is registered, so transformers hands the
    backend mask=None and never builds an N x N mask; a real padding mask is
    caught by the forward guard enable_fa_p100 installs instead;
  * everything the kernel cannot do raises NotImplementedError rather than
    degrading: attention masks, output_attentions, head_mask, sliding windows,
    dropout, head_dim outside {64, 128}, a scale other than 1/sqrt(D), and
    q_len != kv_len (a populated KV cache);
  * fp16 inputs run as they are, and so (beyond the reference) do bf16 ones;
    other dtypes (or a mix) are cast to the autocast dtype under fp16 or bf16
    autocast, and to fp16 with a single warning outside autocast. Outside
    autocast the output is cast back to the input dtype, as the reference does;
    under autocast it keeps the autocast dtype, as SDPA's output does there
    (the reference casts it back to q's dtype, fp32 for Qwen3's normed q, and the
    o_proj that follows casts it down again: the same values, for two extra
    elementwise passes forward and two backward per layer).
"""
import warnings

import torch

from fa_p100 import flash_attn_bnhd

_IMPL_NAME = "fa_p100"
_warned_cast = False


def _unsupported(attention_mask, dropout, scaling, query, key, kwargs):
    """The first reason this call cannot be served, or None."""
    head_dim = query.size(-1)
    if attention_mask is not None:
        return ("fa_p100 got an attention mask, but the kernel takes none; pack "
                "sequences to one length so no padding mask is needed")
    if kwargs.get("output_attentions", False):
        return ("fa_p100 never forms the attention probabilities, so "
                "output_attentions=True is unavailable; use the eager backend")
    if kwargs.get("head_mask") is not None:
        return "fa_p100 does not support head_mask"
    if kwargs.get("sliding_window") is not None:
        return (f"fa_p100 computes dense or causal attention only; this layer asks "
                f"for a sliding window of {kwargs['sliding_window']}")
    if dropout:
        return f"fa_p100 has no attention dropout (got {dropout})"
    if head_dim not in (64, 128):
        return f"fa_p100 needs head_dim 64 or 128, got {head_dim}"
    if scaling is not None and abs(scaling - head_dim ** -0.5) > 1e-6:
        return (f"fa_p100 always scales by 1/sqrt(D) = {head_dim ** -0.5:.6g}; the "
                f"model asks for {scaling:.6g}")
    if key.size(2) != query.size(2):
        return (f"fa_p100 needs equal query and key lengths, got q={query.size(2)} "
                f"kv={key.size(2)}: that is KV-cache decoding, which this training "
                "kernel does not serve")
    return None


def fa_p100_attention_forward(module, query, key, value, attention_mask, dropout=0.0,
                              scaling=None, is_causal=None, **kwargs):
    """transformers attention-interface entry point (fa_p100_hf.py:46-142)."""
    global _warned_cast
    reason = _unsupported(attention_mask, dropout, scaling, query, key, kwargs)
    if reason is not None:
        raise NotImplementedError(reason)

    if is_causal is None:
        is_causal = bool(getattr(module, "is_causal", True)) and query.size(2) > 1

    in_dtype = query.dtype
    autocast = torch.is_autocast_enabled("cuda")
    # fp16 (the reference's type) and bf16 run as they are; anything else (fp32,
    # or a mix -- Qwen3's q/k leave their fp32 RMSNorm weights in fp32 even under
    # autocast) is cast to the autocast dtype when autocast is on, as SDPA's
    # inputs would be, and otherwise to fp16 as the reference does
    native = all(t.dtype == torch.float16 for t in (query, key, value)) or all(
        t.dtype == torch.bfloat16 for t in (query, key, value))
    if not native:
        target = torch.get_autocast_dtype("cuda") if autocast else torch.float16
        if target not in (torch.float16, torch.bfloat16):
            target = torch.float16
        if not autocast and not _warned_cast:
            warnings.warn(
                f"fa_p100: casting q={query.dtype} k={key.dtype} v={value.dtype} to "
                "float16 outside autocast (the kernel computes in fp16 or bf16); wrap "
                "the step in torch.autocast('cuda', torch.float16 or torch.bfloat16)",
                stacklevel=2)
            _warned_cast = True
        query, key, value = query.to(target), key.to(target), value.to(target)

    # output straight in (B, N, H, D), the layout fa_p100_hf.py:142 transposes to
    out = flash_attn_bnhd(query, key, value, causal=bool(is_causal),
                          full_precision=getattr(module, "_fa_p100_full_precision", False))
    # under autocast the output stays in the dtype it was computed in (the
    # consumer, o_proj, runs in that dtype too), as SDPA's does; outside
    # autocast it goes back to the input dtype
    return (out if autocast else out.to(in_dtype)), None


def register():
    """Put "fa_p100" into transformers' attention registry; idempotent."""
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    ALL_ATTENTION_FUNCTIONS[_IMPL_NAME] = fa_p100_attention_forward
    return _IMPL_NAME


def _set_impl(config, name):
    config._attn_implementation = name
    for sub in (getattr(config, "sub_configs", None) or {}):
        child = getattr(config, sub, None)
        if child is not None:
            _set_impl(child, name)


def enable_fa_p100(model, full_precision=False):
    """Route `model`'s attention through the kernels and guard what they cannot do
    (fa_p100_hf.py:161-213). Returns the model."""
    register()
    _set_impl(model.config, _IMPL_NAME)
    for mod in model.modules():
        cfg = getattr(mod, "config", None)
        if cfg is not None and hasattr(cfg, "_attn_implementation"):
            _set_impl(cfg, _IMPL_NAME)
        mod._fa_p100_full_precision = full_precision

    # q_len == kv_len is required, so a KV cache can never be used: default it off.
    model.config.use_cache = False
    if getattr(model, "generation_config", None) is not None:
        model.generation_config.use_cache = False

    if not getattr(model, "_fa_p100_guarded", False):
        wrapped = model.forward

        def guarded_forward(*args, attention_mask=None, use_cache=None, **kwargs):
            # transformers drops the mask before the attention call for a backend
            # with no mask function, so this is the last place to catch padding.
            if attention_mask is not None and not bool(attention_mask.all()):
                raise NotImplementedError(
                    "fa_p100 cannot apply a padding mask and transformers would drop "
                    "it without a word; pack the batch so every position is real")
            # Raised here, before prefill, not at the first decode step.
            if use_cache:
                raise NotImplementedError(
                    "fa_p100 needs q_len == kv_len and so cannot use a KV cache; for "
                    "cache-free generation set generation_config.use_cache = False")
            return wrapped(*args, attention_mask=attention_mask, use_cache=use_cache, **kwargs)

        model.forward = guarded_forward
        model._fa_p100_guarded = True
    return model

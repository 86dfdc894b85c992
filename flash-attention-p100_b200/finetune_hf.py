"""Fine-tune throughput harness: the same short fine-tune run twice -- once
with torch SDPA attention, once through the B200 kernels registered as
"fa_p100" -- from the same initial weights, over the same token blocks in the
same order. It reports both loss trajectories (does training through the
kernels follow the same curve?) and the median step time and peak memory (is it
faster?). This is the method of the reference's finetune_hf.py:90-127; its
chunked language-model-head loss (:45-70) is reproduced because at long
sequences the 151936-entry vocabulary, not attention, would otherwise dominate
memory.

Offline here there is no checkpoint, tokenizer or corpus, so by default the
model is a randomly initialised Qwen3 with Qwen3-0.6B's architecture and the
data are packed blocks of uniformly drawn token ids. --model (a Hugging Face id
or local path) and --corpus (a text file, tokenised with the model's
tokenizer) switch to the real ones where they exist.

Precision: fp32 master weights, autocast to fp16 (the reference's Pascal
constraint) or bf16 (--dtype bf16, native on B200), a GradScaler for fp16.

    python finetune_hf.py --steps 20 --seq-len 8192            # synthetic, config 4
    python finetune_hf.py --model Qwen/Qwen3-0.6B --corpus corpus.txt
"""
import argparse
import json
import statistics

import torch


def qwen3_0p6b_config(layers=None, vocab=None):
    """Qwen3-0.6B's architecture (28 decoder layers, hidden 1024, 16 query and 8
    key/value heads of 128, SwiGLU 3072, q/k RMSNorm, RoPE theta 1e6, tied
    151936-entry vocabulary), initialised N(0, 0.02). `layers` / `vocab` shrink
    it for quick checks."""
    from transformers import Qwen3Config
    return Qwen3Config(vocab_size=vocab or 151936, hidden_size=1024, intermediate_size=3072,
                       num_hidden_layers=layers or 28, num_attention_heads=16,
                       num_key_value_heads=8, head_dim=128, max_position_embeddings=40960,
                       initializer_range=0.02, rms_norm_eps=1e-6,
                       rope_parameters={"rope_theta": 1e6, "rope_type": "default"},
                       tie_word_embeddings=True, attn_implementation="sdpa")


def synthetic_blocks(vocab, seq_len, n_blocks, seed=0):
    """(n_blocks, seq_len) token ids drawn uniformly from the vocabulary."""
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n_blocks, seq_len), generator=gen)


def corpus_blocks(path, tokenizer, seq_len, n_blocks):
    """The corpus tokenised and cut into (n_blocks, seq_len) packed blocks: every
    position a real token, so no attention mask is needed."""
    with open(path) as fh:
        ids = tokenizer(fh.read(), return_tensors="pt").input_ids[0]
    if ids.numel() < seq_len * n_blocks:
        raise SystemExit(f"{path}: {ids.numel()} tokens, {seq_len * n_blocks} needed")
    return ids[: seq_len * n_blocks].reshape(n_blocks, seq_len)


def chunked_lm_loss(model, ids, chunks):
    """Mean next-token cross-entropy with the LM head applied chunk by chunk
    under activation checkpointing: the fp32 logits of one chunk exist at a
    time, in the forward and again (recomputed) in the backward."""
    hidden = model.model(input_ids=ids, use_cache=False).last_hidden_state[:, :-1]
    targets = ids[:, 1:]

    def piece(h, t):
        logits = model.lm_head(h).float()
        return torch.nn.functional.cross_entropy(logits.flatten(0, 1), t.flatten(),
                                                 reduction="sum")

    total = None
    for h, t in zip(hidden.chunk(chunks, dim=1), targets.chunk(chunks, dim=1)):
        part = torch.utils.checkpoint.checkpoint(piece, h, t, use_reentrant=False)
        total = part if total is None else total + part
    return total / targets.numel()


def build_model(impl, args, device):
    """Same seed, same weights for both implementations."""
    from transformers import AutoModelForCausalLM, Qwen3ForCausalLM
    torch.manual_seed(0)
    if args.model:
        model = AutoModelForCausalLM.from_pretrained(args.model, dtype=torch.float32,
                                                     attn_implementation="sdpa").to(device)
    else:
        with torch.device(device):
            model = Qwen3ForCausalLM(qwen3_0p6b_config(args.layers, args.vocab))
    model.config.use_cache = False
    if args.grad_checkpointing:
        model.gradient_checkpointing_enable()
    if impl == "fa_p100":
        import fa_p100_hf
        fa_p100_hf.enable_fa_p100(model, full_precision=args.full_precision)
    return model.train()


def run(impl, blocks, args, device):
    """One fine-tune; returns losses, median step time (ms, CUDA events over the
    whole optimizer step) and peak memory (GiB)."""
    model = build_model(impl, args, device)
    opt = torch.optim.AdamW(model.parameters(), lr=args.lr)
    half = torch.float16 if args.dtype == "fp16" else torch.bfloat16
    scaler = torch.amp.GradScaler("cuda", enabled=half == torch.float16)
    torch.cuda.reset_peak_memory_stats(device)
    losses, times = [], []
    for step in range(args.steps):
        batch = blocks[step % blocks.size(0)].unsqueeze(0).to(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        with torch.autocast("cuda", dtype=half):
            loss = chunked_lm_loss(model, batch, args.loss_chunks)
        scaler.scale(loss).backward()
        scaler.step(opt)
        scaler.update()
        opt.zero_grad(set_to_none=True)
        end.record()
        end.synchronize()
        losses.append(float(loss.item()))
        if step >= args.warmup:      # the first steps build autograd state
            times.append(start.elapsed_time(end))
        if args.verbose:
            print(f"  [{impl}] step {step:3d}  loss {losses[-1]:.4f}  "
                  f"{start.elapsed_time(end):8.1f} ms", flush=True)
    peak = torch.cuda.max_memory_allocated(device) / 2**30
    del model, opt
    torch.cuda.empty_cache()
    return {"impl": impl, "losses": losses,
            "median_step_ms": statistics.median(times) if times else float("nan"),
            "peak_gib": peak}


def compare(args, device="cuda"):
    """Both runs, sdpa first; returns the summary dict the CLI prints."""
    import fa_p100_hf
    fa_p100_hf.register()
    if args.corpus:
        from transformers import AutoTokenizer
        if not args.model:
            raise SystemExit("--corpus needs --model (its tokenizer)")
        blocks = corpus_blocks(args.corpus, AutoTokenizer.from_pretrained(args.model),
                               args.seq_len, args.blocks)
    else:
        vocab = args.vocab or 151936
        blocks = synthetic_blocks(vocab, args.seq_len, args.blocks)
    results = [run(impl, blocks, args, device) for impl in ("sdpa", "fa_p100")]
    sdpa, ours = results
    drift = max(abs(a - b) for a, b in zip(sdpa["losses"], ours["losses"]))
    return {"args": vars(args), "results": results,
            "speedup": sdpa["median_step_ms"] / ours["median_step_ms"],
            "memory_ratio": ours["peak_gib"] / sdpa["peak_gib"],
            "max_loss_difference": drift}


def parser():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--model", default=None, help="HF id or path (default: random-init Qwen3-0.6B shape)")
    ap.add_argument("--corpus", default=None, help="text file (default: synthetic token blocks)")
    ap.add_argument("--seq-len", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--blocks", type=int, default=8)
    ap.add_argument("--lr", type=float, default=1e-5)
    ap.add_argument("--loss-chunks", type=int, default=8)
    ap.add_argument("--layers", type=int, default=None, help="decoder layers (synthetic model)")
    ap.add_argument("--vocab", type=int, default=None, help="vocabulary size (synthetic model)")
    ap.add_argument("--dtype", choices=("fp16", "bf16"), default="fp16")
    ap.add_argument("--grad-checkpointing", action="store_true")
    ap.add_argument("--full-precision", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--out", default=None)
    return ap


def main(argv=None):
    args = parser().parse_args(argv)
    summary = compare(args)
    print(f"{'':<10}{'median step':>14}{'peak mem':>12}{'final loss':>13}")
    for r in summary["results"]:
        print(f"{r['impl']:<10}{r['median_step_ms']:>11.1f} ms{r['peak_gib']:>9.2f} GiB"
              f"{r['losses'][-1]:>13.4f}")
    print(f"speedup {summary['speedup']:.3f}x   memory {summary['memory_ratio']:.2f}x of sdpa   "
          f"max |loss difference| {summary['max_loss_difference']:.2e}")
    if args.out:
        with open(args.out, "w") as fh:
            json.dump(summary, fh, indent=2)
    return summary


if __name__ == "__main__":
    main()

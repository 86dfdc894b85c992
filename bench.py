#!/usr/bin/env python
"""Attention fwd+bwd benchmark (BASELINE.json metric: attention fwd+bwd TFLOPS per
GPU and % of the fp16 tensor peak; Qwen3-0.6B-shaped step ms).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload C3a|...] [--ring]

One step = one forward + one backward of the attention hot path over one batch
of seeded synthetic fp16 inputs (i.i.d. N(0,1), x0.5 for config 3, as
BASELINE.json's configs say). The default workload is C3a causal (B=4, Hq=32,
Hkv=8, N=3000, D=128): the largest single-GPU attention configuration.

Our arm (--impl ours), one JSON line from rank 0:
  value     whole-job TFLOPS with inputs resident in HBM, through the C ABI
            (fa_b200_forward_strided + fa_b200_backward_stages), L2 flushed
            (256 MiB write) between steps, outside the timed events;
  e2e       the same metric through the public API (fa_p100.flash_attn +
            autograd backward) with q, k, v, dO copied from pinned host memory
            and dq, dk, dv copied back inside the timed region, every step;
            uploads and read-backs run on two copy streams, overlapping the
            neighbouring steps' compute as a training input pipeline does;
  roofline  the dominant kernel's algorithmic FLOPs (or bytes) / its CUDA-event
            time, against MEASURED_PEAKS.json;
  sdpa      torch fp16 scaled_dot_product_attention fwd+bwd on the same inputs,
            same L2 flush and CUDA events (the reference's own comparison,
            bench_train.py:24-58);
  north_star, c1, c2, c3a_noncausal, c3b, c3b_noncausal, qwen3_layer   the
            same measurement (ours and SDPA) at (1,32,8192,128) causal, C1, C2,
            C3a non-causal, C3b (MQA, ragged N) both ways and the Qwen3 layer
            shape (N=1 only);
  qwen3_0p6b_step_ms   BASELINE config 4 through the HF registration vs SDPA;
  cpu_baseline  the reference's CPU path (torch fp32 eager attention, restated
            in oracle/) on one (batch, kv-head) group of the workload,
            extrapolated to the whole workload by FLOPs (rank 0, N=1).
Multi-GPU (torchrun, N>1): `value` is N data-parallel replicas -- every rank
runs its own C3a batch, no collective on the data path (weak scaling), time =
max over ranks; `ring_c5` is BASELINE config 5 (B=1, Hq=32, Hkv=8, N=131072)
zigzag-sharded over the N ranks with ring context parallelism (NCCL
send/recv of K/V and the travelling dK/dV accumulators, strong scaling), its
efficiency measured against the same problem on one GPU in the same job.

The reference arm (--impl reference) times the reference's CPU implementation
of the path (fa_p100.reference, restated in oracle/attention_oracle.py) on the
host cores, rank 0 only.
"""
import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "flash-attention-p100_b200")
for _p in (PKG, ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "attn fwd+bwd TFLOPS/GPU & % of fp16 tensor peak; Qwen3-0.6B-shape step ms"
UNIT = "TFLOPS"
WORKLOADS = {
    # name: (B, Hq, Hkv, N, D, causal, input scale)
    "C1": (1, 16, 16, 2048, 64, True, 1.0),
    "C2": (1, 8, 8, 4096, 128, True, 1.0),
    "C3a": (4, 32, 8, 3000, 128, True, 0.5),
    "C3a_noncausal": (4, 32, 8, 3000, 128, False, 0.5),
    "C3b": (2, 16, 1, 1537, 64, True, 0.5),
    "C3b_noncausal": (2, 16, 1, 1537, 64, False, 0.5),
    "north_star": (1, 32, 32, 8192, 128, True, 1.0),
    "qwen3_layer": (1, 16, 8, 8192, 128, True, 1.0),
    "C5": (1, 32, 8, 131072, 128, True, 1.0),
}
# measured beside the headline at N=1 (key in the JSON line: workload)
SIDE_WORKLOADS = {"north_star": "north_star", "c1": "C1", "c2": "C2",
                  "c3a_noncausal": "C3a_noncausal", "c3b": "C3b", "c3b_noncausal": "C3b_noncausal",
                  "qwen3_layer": "qwen3_layer"}
FALLBACK_PEAK_TFLOPS = 1590.0
L2_FLUSH_BYTES = 256 << 20
FLOP_CONVENTION = "fwd 4*B*Hq*D*pairs (causal pairs N(N+1)/2), fwd+bwd 3.5x"


def flops_fwd(B, Hq, N, D, causal):
    pairs = N * (N + 1) / 2 if causal else float(N) * N
    return 4.0 * B * Hq * D * pairs


def step_flops(workload):
    B, Hq, Hkv, N, D, causal, _ = WORKLOADS[workload]
    return 3.5 * flops_fwd(B, Hq, N, D, causal)


def load_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return float(pk["bf16_tflops"]), float(pk["hbm_gbs"]), "measured (MEASURED_PEAKS.json, burst)"
    except (OSError, KeyError, ValueError):
        return FALLBACK_PEAK_TFLOPS, 6650.0, "fallback"


def load_traffic(workload):
    """dram bytes per launch of each kernel, from a committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(workload, {})
    except (OSError, ValueError):
        return {}


class ClockSampler:
    """Samples SM clock and clock-event reasons with NVML while running."""

    REASONS = {
        "sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, device_indices, period_s=0.005):
        self.period = period_s
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._handles = [pynvml.nvmlDeviceGetHandleByIndex(i) for i in device_indices]
            self.max_mhz = max(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
                               for h in self._handles)
        except Exception:  # NVML unavailable: report no clock data
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            for h in self._handles:
                try:
                    mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    util = nv.nvmlDeviceGetUtilizationRates(h).gpu
                    reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((mhz, util, reasons))
                except Exception:
                    pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [],
                    "samples": 0, "source": "nvml unavailable"}
        loaded = [s for s in self.samples if s[1] > 0] or self.samples
        reasons = set()
        for _, _, r in loaded:
            for name, bit in self.REASONS.items():
                if r & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[0] for s in loaded), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.samples),
                "samples_under_load": len(loaded), "source": "nvml"}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(x, world, device):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ---------------------------------------------------------------------------
# CPU side: the reference's path on the host cores (bounded sample)
# ---------------------------------------------------------------------------
def cpu_sample_shape(workload):
    """One (batch, kv-group) slice of the workload: the GQA group of query heads
    that share kv head 0, at the full sequence length."""
    B, Hq, Hkv, N, D, causal, sc = WORKLOADS[workload]
    return 1, Hq // Hkv, 1, N, D, causal, sc


def cpu_step(workload, steps, warmup, min_seconds=0.0):
    """The CPU reference step on one (batch, kv-head) group of `workload`.
    Returns (TFLOPS, extrapolated whole-workload ms per step, threads, sample
    description); the slice's TFLOPS stands for the whole workload's, whose
    time is extrapolated by FLOPs."""
    from oracle import attention_oracle as orc
    torch.set_num_threads(os.cpu_count() or 1)
    B, Hq, Hkv, N, D, causal, sc = cpu_sample_shape(workload)
    q, k, v, do = orc.seeded_inputs(B, Hq, Hkv, N, D, seed=7, scale=sc)
    for _ in range(warmup):
        orc.reference_step(q, k, v, do, causal)
    times = []
    while len(times) < steps or (sum(times) < min_seconds and len(times) < 200):
        t0 = time.perf_counter()
        orc.reference_step(q, k, v, do, causal)
        times.append(time.perf_counter() - t0)
    fl = 3.5 * flops_fwd(B, Hq, N, D, causal)
    ms_slice = statistics.median(times) * 1e3
    tflops = fl / (ms_slice * 1e-3) / 1e12
    ms_full = ms_slice * step_flops(workload) / fl
    sample = (f"one (batch, kv-head) group of {workload} ({Hq} q heads / 1 kv head, N={N}, D={D}, "
              f"causal={causal}), median of {len(times)} steps of {ms_slice:.1f} ms: torch fp32 "
              f"eager fwd+bwd (fa_p100.reference formula) on the host; whole-workload time "
              f"extrapolated by FLOPs")
    return tflops, ms_full, torch.get_num_threads(), sample


def run_reference(args, world, rank):
    if rank != 0:
        return 0
    value, ms, cores, sample = cpu_step(args.workload, args.steps, args.warmup)
    B, Hq, Hkv, N, D, causal, _ = WORKLOADS[args.workload]
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "B": B, "Hq": Hq, "Hkv": Hkv, "N": N, "D": D,
                   "causal": causal, "sample": sample, "flop_convention": FLOP_CONVENTION},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# GPU side: our kernels
# ---------------------------------------------------------------------------
STAGE_ROWSUM, STAGE_DKDV, STAGE_DQ, STAGE_FUSED = 1, 2, 4, 8
# The default backward for the reference's contract (fp32 dq): the row-sum
# preprocess (which also zeroes dq) and the fused dK/dV/dQ kernel (plus, for a
# GQA group split over CTAs, its dK/dV accumulator conversion). --deterministic
# times the bitwise-reproducible backward instead: fp16 dq from the dK/dV and dQ
# kernels.
PATHS = {
    "fused": (("fwd", "bwd_rowsum", "bwd_fused"), (STAGE_ROWSUM, STAGE_FUSED), 1),
    "deterministic": (("fwd", "bwd_rowsum", "bwd_dkdv", "bwd_dq"),
                      (STAGE_ROWSUM, STAGE_DKDV, STAGE_DQ), 0),
}


def kernel_work(name, B, Hq, Hkv, N, D, causal):
    """Algorithmic work of one launch: (amount, unit, bound).
    fwd: the forward's 2 contractions; fused: the backward's 5 (S recompute,
    dP, dV, dK, dQ); rowsum: bytes of O and dO read, Dv and LSE*log2e written,
    and the fp32 dq zeroed."""
    ff = flops_fwd(B, Hq, N, D, causal)
    if name == "fwd":
        return ff, "TFLOP/s", "tensor"
    if name == "bwd_fused":
        return 2.5 * ff, "TFLOP/s", "tensor"
    if name == "bwd_dkdv":
        return 2.0 * ff, "TFLOP/s", "tensor"
    if name == "bwd_dq":
        return 0.5 * ff, "TFLOP/s", "tensor"
    return 2.0 * B * Hq * N * D * 2 + 2 * B * Hq * N * 4 + B * Hq * N * D * 4, "GB/s", "hbm"


def seeded_device_inputs(workload, dev, seed):
    B, Hq, Hkv, N, D, causal, sc = WORKLOADS[workload]
    gen = torch.Generator(device=dev).manual_seed(seed)

    def rnd(h):
        return (torch.randn(B, h, N, D, device=dev, generator=gen) * sc).half()

    return rnd(Hq), rnd(Hkv), rnd(Hkv), rnd(Hq)


def split_group(lib, B, Hq, Hkv, N, D, causal):
    """Whether the fused backward splits a GQA group (it then adds the dK/dV
    accumulator conversion launch), as the library plans it for the workspace
    the bench gives it."""
    import ctypes
    import _lib
    gsplit, hg = ctypes.c_int(0), ctypes.c_int(0)
    ws = lib.fa_b200_backward_workspace_bytes_gqa(B, Hq, Hkv, N, D)
    _lib.check(lib.fa_b200_backward_plan(B, Hq, Hkv, N, D, int(causal), ws, ctypes.byref(gsplit),
                                         ctypes.byref(hg)), "fa_b200_backward_plan")
    return gsplit.value > 1


def queue_ahead(cycles=200_000):
    """A ~0.1 ms spin on the GPU before a timed step, outside its events: the
    host enqueues the whole step meanwhile, so at small sizes (C1's step is
    ~0.09 ms) the events time the kernels, not host launch gaps between them."""
    torch.cuda._sleep(cycles)


def time_kernels(lib, dev, workload, q, k, v, do, steps, warmup, flush, deterministic=False,
                 clocks=None, world=1):
    """Our kernels on resident inputs through the C ABI: per step one forward,
    the row-sum preprocess and the fused backward (or, deterministic, the dK/dV
    and dQ kernels), CUDA events on the launching stream around each launch, L2
    flushed between steps outside the events. Returns (ms per step, {kernel: ms})."""
    import _lib
    B, Hq, Hkv, N, D, causal, _ = WORKLOADS[workload]
    o = torch.empty_like(q)
    lse = torch.empty(B, Hq, N, device=dev)
    kernels, stages, dq_fp32 = PATHS["deterministic" if deterministic else "fused"]
    dq = torch.empty(q.shape, device=dev, dtype=torch.float32 if dq_fp32 else torch.float16)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    ws_bytes = lib.fa_b200_backward_workspace_bytes_gqa(B, Hq, Hkv, N, D)
    ws = torch.empty(ws_bytes // 4, device=dev)
    sq, skv = _lib.strides_of(q), _lib.strides_of(k)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    step_ev = []

    def step(record):
        nk = len(kernels)
        marks = [torch.cuda.Event(enable_timing=True) for _ in range(nk + 1)] if record else None
        if record:
            marks[0].record(stream)
        st = lib.fa_b200_forward_strided(q.data_ptr(), sq, k.data_ptr(), skv, v.data_ptr(), skv,
                                         o.data_ptr(), sq, lse.data_ptr(), B, Hq, Hkv, N, D,
                                         _lib.DTYPE_FP16, int(causal), 0, sp)
        _lib.check(st, "fa_b200_forward_strided")
        for i, mask in enumerate(stages):
            if record:
                marks[i + 1].record(stream)
            st = lib.fa_b200_backward_stages(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), o.data_ptr(),
                lse.data_ptr(), dq.data_ptr(), dq_fp32, dk.data_ptr(), dv.data_ptr(),
                ws.data_ptr(), ws_bytes, B, Hq, Hkv, N, D, int(causal), mask, sp)
            _lib.check(st, "fa_b200_backward_stages")
        if record:
            marks[nk].record(stream)
            step_ev.append(marks)

    for _ in range(warmup):
        flush.fill_(1.0)
        step(False)
    torch.cuda.synchronize(dev)
    if _lib.device_error(dev.index) != 0:
        raise RuntimeError(f"device error word set during the {workload} warm-up")
    ctx = clocks if clocks is not None else _Null()
    with ctx:
        barrier(world)
        torch.cuda.synchronize(dev)
        for _ in range(steps):
            flush.fill_(1.0)   # L2 flush, outside the step's events
            queue_ahead()
            step(True)
        torch.cuda.synchronize(dev)
        barrier(world)
    if _lib.device_error(dev.index) != 0:
        raise RuntimeError(f"device error word set during the {workload} timed steps")
    per_kernel = {n: 0.0 for n in kernels}
    total = 0.0
    for m in step_ev:
        for i, n in enumerate(kernels):
            per_kernel[n] += m[i].elapsed_time(m[i + 1])
        total += m[0].elapsed_time(m[len(kernels)])
    return total / steps, {n: t / steps for n, t in per_kernel.items()}


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


def time_sdpa(dev, workload, q, k, v, do, steps, warmup, flush):
    """torch fp16 scaled_dot_product_attention fwd+bwd (torch's default SDPA
    dispatch, GQA through enable_gqa) on the same inputs, L2 flushed between
    steps outside the events. Returns ms per step."""
    import torch.nn.functional as F
    causal = WORKLOADS[workload][5]
    gqa = q.size(1) != k.size(1)
    qs, ks, vs = (t.detach().clone().requires_grad_(True) for t in (q, k, v))

    def step():
        for t in (qs, ks, vs):
            t.grad = None
        out = F.scaled_dot_product_attention(qs, ks, vs, is_causal=causal, enable_gqa=gqa)
        out.backward(do)

    for _ in range(warmup):
        flush.fill_(1.0)
        step()
    torch.cuda.synchronize(dev)
    total = 0.0
    for _ in range(steps):
        flush.fill_(1.0)
        queue_ahead()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        step()
        b.record()
        b.synchronize()
        total += a.elapsed_time(b)
    del qs, ks, vs
    return total / steps


def kernel_report(workload, per_kernel, peak_tf, peak_gbs, peak_src):
    """Per-kernel achieved rates and the roofline of the dominant kernel."""
    B, Hq, Hkv, N, D, causal, _ = WORKLOADS[workload]
    kernels = {}
    for n, ms in per_kernel.items():
        w, u, _ = kernel_work(n, B, Hq, Hkv, N, D, causal)
        kernels[n] = {"ms": ms, "achieved": w / (ms * 1e-3) / (1e12 if u == "TFLOP/s" else 1e9),
                      "unit": u}
    dom = max(per_kernel, key=per_kernel.get)
    work, unit, bound = kernel_work(dom, B, Hq, Hkv, N, D, causal)
    achieved = kernels[dom]["achieved"]
    peak = peak_tf if unit == "TFLOP/s" else peak_gbs
    roofline = {"kernel": dom, "bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                "frac": achieved / peak, "traffic": load_traffic(workload).get(dom),
                "algorithmic_per_launch": work, "peak_source": peak_src}
    return kernels, roofline


def side_measurement(lib, dev, workload, steps, warmup, flush, peaks, seed=4321):
    """Our kernels and SDPA at one more workload: value, % of peak, per-kernel
    rates, roofline and the SDPA comparison."""
    peak_tf, peak_gbs, peak_src = peaks
    B, Hq, Hkv, N, D, causal, sc = WORKLOADS[workload]
    q, k, v, do = seeded_device_inputs(workload, dev, seed)
    ms, per_kernel = time_kernels(lib, dev, workload, q, k, v, do, steps, warmup, flush)
    sd_ms = time_sdpa(dev, workload, q, k, v, do, steps, warmup, flush)
    fl = step_flops(workload)
    value = fl / (ms * 1e-3) / 1e12
    kernels, roofline = kernel_report(workload, per_kernel, peak_tf, peak_gbs, peak_src)
    del q, k, v, do
    torch.cuda.empty_cache()
    return {"workload": workload, "B": B, "Hq": Hq, "Hkv": Hkv, "N": N, "D": D, "causal": causal,
            "value": value, "unit": UNIT, "ms_per_step": ms,
            "pct_of_peak": 100.0 * value / peak_tf, "kernels": kernels, "roofline": roofline,
            "sdpa": {"value": fl / (sd_ms * 1e-3) / 1e12, "ms_per_step": sd_ms},
            "vs_sdpa": sd_ms / ms}


def qwen3_step_ms(dev, attn, steps, warmup, seq=8192):
    """a Qwen3-0.6B-shaped decoder (28 layers, hidden 1024,
    16 query / 8 kv heads of 128, q/k RMSNorm, RoPE theta 1e6, SwiGLU 3072,
    vocab 151936 tied), random init N(0, 0.02), token ids uniform in the vocab,
    B=1, `seq` tokens, one fp16-autocast forward + backward with the model's
    own next-token cross-entropy. attn = "fa_p100" (the HF registration) or
    "sdpa". Returns the median step time in ms (CUDA events)."""
    from transformers import Qwen3Config, Qwen3ForCausalLM
    import fa_p100_hf
    cfg = Qwen3Config(vocab_size=151936, hidden_size=1024, intermediate_size=3072,
                      num_hidden_layers=28, num_attention_heads=16, num_key_value_heads=8,
                      head_dim=128, max_position_embeddings=40960, initializer_range=0.02,
                      rope_parameters={"rope_theta": 1e6, "rope_type": "default"},
                      tie_word_embeddings=True, attn_implementation="sdpa")
    torch.manual_seed(0)
    with torch.device(dev):
        model = Qwen3ForCausalLM(cfg)
    if attn == "fa_p100":
        fa_p100_hf.enable_fa_p100(model)
    gen = torch.Generator(device=dev).manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (1, seq), device=dev, generator=gen)

    def step():
        model.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.float16):
            loss = model(input_ids=ids, labels=ids).loss
        loss.backward()
        return loss

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    times = []
    for _ in range(steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        loss = step()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b))
    if not torch.isfinite(loss).item():
        raise RuntimeError(f"qwen3 step ({attn}) produced a non-finite loss")
    del model
    torch.cuda.empty_cache()
    return statistics.median(times), float(loss.item())


def run_ours(args, world, rank, local):
    import _lib
    import fa_p100

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    lib = _lib.lib()
    peaks = load_peak()
    peak_tf, peak_gbs, peak_src = peaks
    B, Hq, Hkv, N, D, causal, sc = WORKLOADS[args.workload]
    gen = torch.Generator(device="cpu").manual_seed(1234 + rank)

    def rnd(h):
        return (torch.randn(B, h, N, D, generator=gen) * sc).half()

    q_h, k_h, v_h, do_h = rnd(Hq), rnd(Hkv), rnd(Hkv), rnd(Hq)
    q, k, v, do = (t.to(dev) for t in (q_h, k_h, v_h, do_h))
    flush = torch.empty(L2_FLUSH_BYTES // 4, device=dev)
    n_kernels = 4 if args.deterministic else 3
    split = not args.deterministic and split_group(lib, B, Hq, Hkv, N, D, causal)

    with ClockSampler([local]) as clocks:
        ms, per_kernel = time_kernels(lib, dev, args.workload, q, k, v, do, args.steps,
                                      args.warmup, flush, args.deterministic, None, world)
    ms = max_over_ranks(ms, world, dev)
    launches = (n_kernels + (1 if split else 0)) * args.steps

    # e2e: public API, host buffers, copies inside the timed region. Laid out
    # like a training input pipeline: step s+1's inputs go up on a copy stream
    # while step s computes, and step s's gradients come back on another copy
    # stream while step s+1 computes (PCIe carries both directions at once).
    # Every step's uploads and read-backs lie inside the timed region, which
    # opens before the first upload and closes after the last read-back; the
    # inputs (q, k, v, dO) are larger than L2 and alternate between two device
    # buffers.
    pin = [t.pin_memory() for t in (q_h, k_h, v_h, do_h)]
    outs_h = [torch.empty(t.shape, dtype=torch.float16).pin_memory() for t in (q_h, k_h, v_h)]
    stream = torch.cuda.current_stream(dev)
    s_up, s_down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    dbuf = [[torch.empty_like(t) for t in (q, k, v, do)] for _ in range(2)]
    up_done = [torch.cuda.Event() for _ in range(2)]
    used = [torch.cuda.Event() for _ in range(2)]

    def upload(j):
        s_up.wait_event(used[j])          # the step that last read buffer j is done
        with torch.cuda.stream(s_up):
            for d, h in zip(dbuf[j], pin):
                d.copy_(h, non_blocking=True)
        up_done[j].record(s_up)

    def e2e_run(n_steps):
        upload(0)
        for st in range(n_steps):
            j = st & 1
            if st + 1 < n_steps:
                upload(j ^ 1)
            stream.wait_event(up_done[j])
            qd, kd, vd = (t.detach().requires_grad_(True) for t in dbuf[j][:3])
            out = fa_p100.flash_attn(qd, kd, vd, causal)
            out.backward(dbuf[j][3])
            used[j].record(stream)
            s_down.wait_event(used[j])
            with torch.cuda.stream(s_down):
                for h, t in zip(outs_h, (qd.grad, kd.grad, vd.grad)):
                    t.record_stream(s_down)
                    h.copy_(t, non_blocking=True)
            del qd, kd, vd, out
        stream.wait_stream(s_down)

    e2e_run(args.warmup)
    torch.cuda.synchronize(dev)
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for ev in used:                       # nothing uploads before the region opens
        ev.record(stream)
    e2e_run(args.steps)
    b.record(stream)
    b.synchronize()
    e2e_ms = a.elapsed_time(b)
    barrier(world)
    launches += (4 if split else 3) * args.steps   # forward, row-sum, fused backward (+ convert)
    e2e_ms = max_over_ranks(e2e_ms / args.steps, world, dev)
    fa_p100.check_device_errors(dev)

    fl = step_flops(args.workload)
    value = world * fl / (ms * 1e-3) / 1e12
    e2e_value = world * fl / (e2e_ms * 1e-3) / 1e12
    kernels, roofline = kernel_report(args.workload, per_kernel, peak_tf, peak_gbs, peak_src)

    # same-run SDPA comparison on the same inputs
    sd_ms = max_over_ranks(time_sdpa(dev, args.workload, q, k, v, do, args.steps, args.warmup,
                                     flush), world, dev)
    del q, k, v, do, pin, outs_h
    torch.cuda.empty_cache()

    ring = None
    if world > 1 and not args.no_ring:
        ring = ring_c5(args, world, rank, local, flush)

    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 (fp32 accumulate)", "data": "synthetic",
        "pct_of_peak": 100.0 * value / world / peak_tf,
        "peak_tflops": peak_tf, "peak_source": peak_src,
        "config": {"workload": args.workload, "B": B, "Hq": Hq, "Hkv": Hkv, "N": N, "D": D,
                   "causal": causal, "inputs": f"N(0,1)*{sc} fp16, seeded",
                   "l2": "flushed (256 MiB write) between steps, outside the timed events",
                   "parallelism": (f"data-parallel replicas x{world}: each rank runs its own "
                                   f"{args.workload} batch, no collective (weak scaling)")
                   if world > 1 else "single GPU",
                   "backward": ("deterministic (fp16 dq, dK/dV + dQ kernels)" if args.deterministic
                                else "fused (fp32 dq, TMA reduce-adds)"),
                   "flops_per_step_per_gpu": fl, "flop_convention": FLOP_CONVENTION},
        "e2e": {"value": e2e_value, "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": sum(t.numel() * 2 for t in (q_h, k_h, v_h, do_h)),
                "d2h_bytes_per_step": sum(t.numel() * 2 for t in (q_h, k_h, v_h)),
                "path": "fa_p100.flash_attn + autograd backward, pinned host buffers, "
                        "uploads and read-backs on copy streams overlapping neighbouring steps"},
        "roofline": roofline,
        "kernels": kernels,
        "sdpa": {"value": world * fl / (sd_ms * 1e-3) / 1e12, "ms_per_step": sd_ms,
                 "what": "torch fp16 F.scaled_dot_product_attention fwd+bwd (default dispatch, "
                         "enable_gqa), same inputs, L2 flush and events"},
        "vs_sdpa": sd_ms / ms,
        "gpu_launches": launches,
        "clocks": clocks.summary(),
    }
    if ring is not None:
        line["ring_c5"] = ring
    if world == 1 and not args.no_side:
        for key, wl in SIDE_WORKLOADS.items():
            line[key] = side_measurement(lib, dev, wl, args.steps, args.warmup, flush, peaks)
    if world == 1 and not args.no_qwen3:
        q_ms, q_loss = qwen3_step_ms(dev, "fa_p100", 5, 3)
        s_ms, s_loss = qwen3_step_ms(dev, "sdpa", 5, 3)
        line["qwen3_0p6b_step_ms"] = {
            "value": q_ms, "sdpa_ms": s_ms, "loss": q_loss, "sdpa_loss": s_loss,
            "config": "BASELINE config 4: 28 layers, hidden 1024, 16/8 heads x 128, seq 8192, "
                      "B=1, fp16 autocast fwd+bwd, random init, attention via fa_p100 registration"}
    if world == 1 and not args.no_cpu_baseline:
        cpu_tf, cpu_ms, cores, sample = cpu_step(args.workload, 3, 1, min_seconds=10.0)
        line["cpu_baseline"] = {"value": cpu_tf, "unit": UNIT, "cores": cores, "kind": "port",
                                "ms_per_step_extrapolated": cpu_ms, "sample": sample}
    print(json.dumps(line), flush=True)
    return 0


def ring_step_fn(world, dev, q, k, v, do):
    import fa_b200_ring as ring
    import fa_p100

    def step():
        for t in (q, k, v):
            t.grad = None
        o = ring.ring_flash_attn(q, k, v) if world > 1 else fa_p100.flash_attn(q, k, v, True)
        o.backward(do)
    return step


def time_ring(world, rank, local, steps, warmup, flush, single=False):
    """Config 5 fwd+bwd: zigzag ring over `world` ranks, or (single) the whole
    sequence through the single-GPU kernels on this rank. Returns ms per step."""
    dev = torch.device("cuda", local)
    B, Hq, Hkv, N, D, causal, sc = WORKLOADS["C5"]
    w = 1 if single else world
    gen = torch.Generator(device=dev).manual_seed(100 + (0 if single else rank))
    n_loc = N // w

    def rnd(h):
        return (torch.randn(B, h, n_loc, D, device=dev, generator=gen) * sc).half()

    q, k, v, do = rnd(Hq).requires_grad_(True), rnd(Hkv).requires_grad_(True), \
        rnd(Hkv).requires_grad_(True), rnd(Hq)
    step = ring_step_fn(w, dev, q, k, v, do)
    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    if not single:
        barrier(world)
    total = 0.0
    for _ in range(steps):
        flush.fill_(1.0)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        step()
        b.record()
        b.synchronize()
        total += a.elapsed_time(b)
    if not single:
        barrier(world)
    del q, k, v, do
    torch.cuda.empty_cache()
    return total / steps


def ring_c5(args, world, rank, local, flush):
    """BASELINE config 5 on the job's ranks (ring context parallelism) and, on
    rank 0, on one GPU; strong-scaling efficiency = t1 / (world * t_world)."""
    import fa_p100
    dev = torch.device("cuda", local)
    steps, warmup = min(args.steps, 5), max(3, min(args.warmup, 3))
    with ClockSampler([local]) as clocks:
        ms = max_over_ranks(time_ring(world, rank, local, steps, warmup, flush), world, dev)
    fa_p100.check_device_errors(dev)
    t1 = None
    if rank == 0:
        t1 = time_ring(world, rank, local, steps, warmup, flush, single=True)
        fa_p100.check_device_errors(dev)
    barrier(world)
    B, Hq, Hkv, N, D, causal, _ = WORKLOADS["C5"]
    total = step_flops("C5")
    if rank != 0:
        return None
    peak_tf, _, _ = load_peak()
    return {"workload": "C5", "B": B, "Hq": Hq, "Hkv": Hkv, "N": N, "D": D, "causal": causal,
            "parallelism": f"ring context parallel, zigzag x{world} (NCCL send/recv)",
            "scaling": "strong", "value": total / (ms * 1e-3) / 1e12, "unit": UNIT,
            "ms_per_step": ms, "steps": steps, "warmup": warmup,
            "pct_of_peak_per_gpu": 100.0 * total / (ms * 1e-3) / 1e12 / world / peak_tf,
            "single_gpu_ms_per_step": t1, "efficiency": t1 / (world * ms),
            "l2": "flushed (256 MiB write) before each step", "clocks": clocks.summary()}


def run_ring(args, world, rank, local):
    """Config 5 alone (--ring): the ring over the job's ranks, strong scaling.
    At one GPU the same problem runs through the single-GPU kernels."""
    import fa_p100
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, device=dev)
    with ClockSampler([local]) as clocks:
        ms = max_over_ranks(time_ring(world, rank, local, args.steps, args.warmup, flush),
                            world, dev)
    fa_p100.check_device_errors(dev)
    B, Hq, Hkv, N, D, causal, _ = WORKLOADS["C5"]
    pieces_fwd = 1 + 2 * (world - 1)
    if rank != 0:
        return 0
    peak_tf, _, peak_src = load_peak()
    value = step_flops("C5") / (ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16 (fp32 accumulate)", "data": "synthetic",
        "pct_of_peak": 100.0 * value / world / peak_tf, "peak_tflops": peak_tf,
        "peak_source": peak_src,
        "config": {"workload": "C5", "B": B, "Hq": Hq, "Hkv": Hkv, "N": N, "D": D,
                   "causal": causal, "parallelism": f"ring context parallel, zigzag x{world}"
                   if world > 1 else "single GPU",
                   "l2": "flushed (256 MiB write) before each step"},
        # each piece: one forward launch, and a row-sum + fused backward launch
        "gpu_launches": args.steps * 3 * pieces_fwd if world > 1 else 3 * args.steps,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="C3a")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-side", action="store_true",
                    help="skip the north-star / C1 / C2 / C3a non-causal side measurements")
    ap.add_argument("--no-ring", action="store_true",
                    help="skip the ring_c5 measurement of multi-GPU runs")
    ap.add_argument("--deterministic", action="store_true",
                    help="time the bitwise-reproducible backward (fp16 dq, dK/dV + dQ kernels)")
    ap.add_argument("--ring", action="store_true",
                    help="only config 5 by ring context parallelism over the ranks")
    ap.add_argument("--no-qwen3", action="store_true",
                    help="skip the Qwen3-0.6B-shaped training step (BASELINE config 4)")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    world, rank, local = dist_setup(args) if args.impl == "ours" else (
        int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0)
    try:
        if args.impl == "reference":
            return run_reference(args, world, rank)
        if args.ring:
            return run_ring(args, world, rank, local)
        return run_ours(args, world, rank, local)
    finally:
        if world > 1 and args.impl == "ours":
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())

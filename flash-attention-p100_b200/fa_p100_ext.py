"""The extension ops `forward` / `backward`, same names and contract as the
reference's pybind11 module (fa_p100_ext.cu:144-147), implemented over the C ABI
of libfa_b200.so (include/fa_b200.h).

    forward(q, k, v, causal, full_precision) -> [o, lse]
    backward(q, k, v, dO, o, lse, causal)    -> [dq (fp32), dk, dv]

Validation and messages follow fa_p100_ext.cu:31-35, :55-65, :106-115 and raise
RuntimeError, as TORCH_CHECK does. Outputs and the row-sum workspace are
allocated here with torch on the inputs' device (fa_p100_ext.cu:68-69,
:121-124); kernels run on torch's current CUDA stream rather than the legacy
default stream. There is no CPU path: CPU tensors are rejected.

Where the reference makes every input contiguous (fa_p100_ext.cu:56, :107-108),
these ops hand strided (B, H, N, D) views with a contiguous D axis -- e.g. the
transposed projections an attention layer produces -- straight to the
kernels' tensor maps; only a layout the tensor maps cannot address (an
unaligned base or stride) is copied first.

A kernel that gives up one of its bounded internal waits leaves its outputs
incomplete and sets a device error word. Every op enqueues an asynchronous
read of that word after its launches and raises RuntimeError at the next op
on the device once the read has landed; `check_device_errors()` synchronises
and raises at once.
"""
import math
import threading

import torch

import _lib

_DEVERR = {1: "a TMA producer waited too long for a free slot",
           2: "the MMA issuer waited too long for an operand",
           3: "the softmax / gradient warps waited too long for an MMA",
           4: "an epilogue waited too long",
           5: "dynamic shared memory was not 1024-byte aligned",
           6: "the failure-detection self-test's deliberate timeout"}


def _device_error_message(code):
    return (f"an attention kernel gave up a bounded internal wait (device error {code}: "
            f"{_DEVERR.get(code, 'unknown')}); the outputs of that call are incomplete")


class _ErrorWatch:
    """Per-thread, per-device check of the kernels' error word without
    synchronising.

    After each call's launches the word is copied (fa_b200_device_error_async)
    into a pinned host int on the same stream and an event is recorded; at the
    next call the copy is read if the event has completed, and a set word
    raises RuntimeError there -- what the reference's AT_CUDA_CHECK after each
    launch (fa_p100_ext.cu:81, :140) does for launch failures. Each host thread
    has its own pinned word and event, so threads that drive one device from
    several streams do not overwrite each other's copy."""

    def __init__(self, device):
        self.device = device
        self.word = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.event = None

    def poll(self):
        ev = self.event
        if ev is not None and ev.query():
            self.event = None
            code = int(self.word[0])
            if code:
                self.clear()
                raise RuntimeError(_device_error_message(code))

    def after_launch(self, stream_ptr):
        _lib.check(_lib.lib().fa_b200_device_error_async(self.word.data_ptr(), stream_ptr),
                   "fa_b200_device_error_async")
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self.event = ev

    def clear(self):
        _lib.device_error(self.device.index, reset=True)
        self.word.zero_()
        self.event = None


_local = threading.local()


def _watches():
    d = getattr(_local, "watches", None)
    if d is None:
        d = _local.watches = {}
    return d


def _watch(device):
    ws = _watches()
    w = ws.get(device.index)
    if w is None:
        w = ws[device.index] = _ErrorWatch(device)
    return w


def check_device_errors(device=None):
    """Synchronise `device` (default: the current one) and raise RuntimeError if
    a kernel of this library gave up a bounded wait since the last check; the
    error word is cleared either way."""
    device = torch.device("cuda", torch.cuda.current_device() if device is None
                          else torch.device(device).index or 0)
    code = _lib.device_error(device.index, reset=True)
    w = _watches().get(device.index)
    if w is not None:
        w.word.zero_()
        w.event = None
    if code < 0:
        raise RuntimeError("reading the device error word failed")
    if code:
        raise RuntimeError(_device_error_message(code))


def _check_in(t, name):
    # fa_p100_ext.cu:31-35
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if t.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError(f"{name} must be fp16 (or bf16)")
    if t.dim() != 4:
        raise RuntimeError(f"{name} must be (B, H, N, D)")


def _dtype_code(q, *others):
    """FA_B200_DTYPE_* of q; every other 16-bit tensor of the call must match."""
    for t in others:
        if t.dtype != q.dtype:
            raise RuntimeError(f"all of q, k, v, dO and o must share one dtype; got {q.dtype} "
                               f"and {t.dtype}")
    return _lib.DTYPE_BF16 if q.dtype == torch.bfloat16 else _lib.DTYPE_FP16


def _stream_ptr(device):
    return torch.cuda.current_stream(device).cuda_stream


def _shapes(q, k, v):
    B, H, N, D = q.shape
    Hkv = k.size(1)
    if D not in (64, 128):
        raise RuntimeError(f"head dim must be 64 or 128, got {D}")
    if N <= 0:
        raise RuntimeError("N must be positive")
    if not (Hkv > 0 and H % Hkv == 0):
        raise RuntimeError(
            f"query heads ({H}) must be a multiple of key/value heads ({Hkv})")
    if k.shape != v.shape:
        raise RuntimeError("k and v must match")
    if k.size(0) != B or k.size(2) != N or k.size(3) != D:
        raise RuntimeError("k/v must be (B, Hkv, N, D) matching q's B, N, D")
    return B, H, Hkv, N, D


def _layout(t):
    """(t, its fa_b200_strides), or a contiguous copy of t and its strides when
    the tensor maps cannot address t in place."""
    st = _lib.strides_of(t)
    if st is None:
        t = t.contiguous()
        st = _lib.strides_of(t)
    return t, st


def _out(t, shape, dtype, device, name):
    """A caller-supplied output (any layout the tensor maps accept) or a new
    contiguous one."""
    if t is None:
        t = torch.empty(shape, device=device, dtype=dtype)
    if tuple(t.shape) != tuple(shape) or t.dtype != dtype or t.device != device:
        raise RuntimeError(f"{name} must be a {dtype} tensor of shape {tuple(shape)} on {device}")
    st = _lib.strides_of(t)
    if st is None:
        raise RuntimeError(f"{name}: the D axis must be contiguous and the base and strides "
                           "16-byte aligned")
    return t, st


def forward(q, k, v, causal, full_precision=False, o=None, lse=None):
    """O (B,Hq,N,D) in q's dtype and LSE (B,Hq,N) fp32 (natural log).
    fa_p100_ext.cu:53-83. q, k, v are fp16 (the reference's type) or bf16; `o`
    may supply the output in any layout with a contiguous D axis, `lse` a
    contiguous fp32 (B,Hq,N) buffer."""
    _check_in(q, "q")
    _check_in(k, "k")
    _check_in(v, "v")
    dtype = _dtype_code(q, k, v)
    B, H, Hkv, N, D = _shapes(q, k, v)
    (q, sq), (k, sk), (v, sv) = _layout(q), _layout(k), _layout(v)
    o, so = _out(o, (B, H, N, D), q.dtype, q.device, "o")
    if lse is None:
        lse = torch.empty((B, H, N), device=q.device, dtype=torch.float32)
    elif (tuple(lse.shape) != (B, H, N) or lse.dtype != torch.float32 or lse.device != q.device
          or not lse.is_contiguous()):
        raise RuntimeError(f"lse must be a contiguous float32 tensor of shape {(B, H, N)} on "
                           f"{q.device}")
    lib = _lib.lib()
    watch = _watch(q.device)
    watch.poll()
    with torch.cuda.device(q.device):
        sp = _stream_ptr(q.device)
        st = lib.fa_b200_forward_strided(
            q.data_ptr(), sq, k.data_ptr(), sk, v.data_ptr(), sv, o.data_ptr(), so,
            lse.data_ptr(), B, H, Hkv, N, D, dtype, 1 if causal else 0,
            1 if full_precision else 0, sp)
        _lib.check(st, "fa_b200_forward_strided")
        watch.after_launch(sp)
    return [o, lse]


def backward_into(q, k, v, dO, o, lse, causal, dq_dtype=torch.float32, dq=None, dk=None,
                  dv=None):
    """dq (dq_dtype), dk, dv (q's dtype). fp32 dq (the default, and `backward`)
    runs the fused one-pass backward, whose dq adds are not bitwise
    deterministic; a 16-bit dq (q's dtype) runs the two-kernel backward (dK/dV,
    then dQ), which is. dq, dk, dv may be supplied in any layout with a
    contiguous D axis (new ones are contiguous)."""
    _check_in(q, "q")
    _check_in(dO, "dO")
    # fa_p100_ext.cu:106-115 checks only q and dO; k, v, o and lse are checked
    # here too, because a wrong dtype would be read as garbage by the kernels.
    for t, name in ((k, "k"), (v, "v"), (o, "o")):
        _check_in(t, name)
    if lse.dtype != torch.float32 or not lse.is_cuda:
        raise RuntimeError("lse must be a CUDA fp32 tensor")
    B, H, Hkv, N, D = _shapes(q, k, v)
    if dO.shape != q.shape or o.shape != q.shape or lse.shape != (B, H, N):
        raise RuntimeError("dO and o must match q, and lse must be (B, Hq, N)")
    dtype = _dtype_code(q, k, v, dO, o)
    if dq_dtype not in (torch.float32, q.dtype):
        raise RuntimeError(f"dq_dtype must be float32 or {q.dtype}")
    (q, sq), (k, sk), (v, sv) = _layout(q), _layout(k), _layout(v)
    (dO, sdo), (o, so) = _layout(dO), _layout(o)
    lse = lse.contiguous()
    dq, sdq = _out(dq, (B, H, N, D), dq_dtype, q.device, "dq")
    dk, sdk = _out(dk, (B, Hkv, N, D), q.dtype, q.device, "dk")
    dv, sdv = _out(dv, (B, Hkv, N, D), q.dtype, q.device, "dv")
    lib = _lib.lib()
    ws_bytes = lib.fa_b200_backward_workspace_bytes_gqa(B, H, Hkv, N, D)
    ws = torch.empty((ws_bytes // 4,), device=q.device, dtype=torch.float32)
    watch = _watch(q.device)
    watch.poll()
    with torch.cuda.device(q.device):
        sp = _stream_ptr(q.device)
        st = lib.fa_b200_backward_strided(
            q.data_ptr(), sq, k.data_ptr(), sk, v.data_ptr(), sv, dO.data_ptr(), sdo,
            o.data_ptr(), so, lse.data_ptr(), dq.data_ptr(), sdq,
            1 if dq_dtype == torch.float32 else 0, dk.data_ptr(), sdk, dv.data_ptr(), sdv,
            ws.data_ptr(), ws_bytes, B, H, Hkv, N, D, dtype, 1 if causal else 0, 0, sp)
        _lib.check(st, "fa_b200_backward_strided")
        watch.after_launch(sp)
    return [dq, dk, dv]


def backward_accumulate(q, k, v, dO, o, lse, causal, dq, dk, dv):
    """Adds this call's gradients into fp32 accumulators: dq (B,Hq,N,D), dk,
    dv (B,Hkv,N,D), any layout with a contiguous D axis (views of larger
    accumulators included). One fused pass (FA_B200_STAGE_ACCUMULATE): dQ and
    dK/dV are added by TMA reduce-adds, so nothing is rounded to 16 bits
    between calls. For callers that sum gradients over several calls, as ring
    attention does over its steps. Returns (dq, dk, dv)."""
    for t, name in ((q, "q"), (dO, "dO"), (k, "k"), (v, "v"), (o, "o")):
        _check_in(t, name)
    if lse.dtype != torch.float32 or not lse.is_cuda:
        raise RuntimeError("lse must be a CUDA fp32 tensor")
    B, H, Hkv, N, D = _shapes(q, k, v)
    if dO.shape != q.shape or o.shape != q.shape or lse.shape != (B, H, N):
        raise RuntimeError("dO and o must match q, and lse must be (B, Hq, N)")
    dtype = _dtype_code(q, k, v, dO, o)
    (q, sq), (k, sk), (v, sv) = _layout(q), _layout(k), _layout(v)
    (dO, sdo), (o, so) = _layout(dO), _layout(o)
    lse = lse.contiguous()
    dq, sdq = _out(dq, (B, H, N, D), torch.float32, q.device, "dq")
    dk, sdk = _out(dk, (B, Hkv, N, D), torch.float32, q.device, "dk")
    dv, sdv = _out(dv, (B, Hkv, N, D), torch.float32, q.device, "dv")
    lib = _lib.lib()
    ws_bytes = lib.fa_b200_backward_workspace_bytes(B, H, N)
    ws = torch.empty((ws_bytes // 4,), device=q.device, dtype=torch.float32)
    stages = 1 | 8 | 16   # FA_B200_STAGE_ROWSUM | FUSED | ACCUMULATE
    watch = _watch(q.device)
    watch.poll()
    with torch.cuda.device(q.device):
        sp = _stream_ptr(q.device)
        st = lib.fa_b200_backward_strided(
            q.data_ptr(), sq, k.data_ptr(), sk, v.data_ptr(), sv, dO.data_ptr(), sdo,
            o.data_ptr(), so, lse.data_ptr(), dq.data_ptr(), sdq, 1, dk.data_ptr(), sdk,
            dv.data_ptr(), sdv, ws.data_ptr(), ws_bytes, B, H, Hkv, N, D, dtype,
            1 if causal else 0, stages, sp)
        _lib.check(st, "fa_b200_backward_strided (accumulate)")
        watch.after_launch(sp)
    return dq, dk, dv


def merge_partial(o, lse, o_part, lse_part):
    """In place: o (fp32, B,H,N,D) and lse (fp32, B,H,N) -- attention over one
    set of keys -- absorb o_part (16-bit) and lse_part, the same queries over
    other keys: lse = logaddexp(lse, lse_part), o = o e^(lse_old - lse) +
    o_part e^(lse_part - lse). Views (e.g. half of a longer accumulator) are
    fine."""
    _check_in(o_part, "o_part")
    B, H, N, D = o_part.shape
    if o.dtype != torch.float32 or tuple(o.shape) != (B, H, N, D) or o.device != o_part.device:
        raise RuntimeError("o must be an fp32 tensor shaped like o_part on its device")
    for t, name in ((lse, "lse"), (lse_part, "lse_part")):
        if t.dtype != torch.float32 or tuple(t.shape) != (B, H, N) or t.device != o_part.device:
            raise RuntimeError(f"{name} must be an fp32 (B, H, N) tensor on o_part's device")
    so = _lib.strides_of(o)
    if so is None:
        raise RuntimeError("o: the D axis must be contiguous and the base and strides 16-byte aligned")
    o_part, sop = _layout(o_part)
    sl = _lib.Strides(*lse.stride())
    slp = _lib.Strides(*lse_part.stride())
    dtype = _lib.DTYPE_BF16 if o_part.dtype == torch.bfloat16 else _lib.DTYPE_FP16
    with torch.cuda.device(o.device):
        st = _lib.lib().fa_b200_merge_partial(o.data_ptr(), so, lse.data_ptr(), sl,
                                              o_part.data_ptr(), sop, lse_part.data_ptr(), slp,
                                              B, H, N, D, dtype, _stream_ptr(o.device))
    _lib.check(st, "fa_b200_merge_partial")
    return o, lse


def backward(q, k, v, dO, o, lse, causal):
    """dq fp32 (B,Hq,N,D), dk, dv in q's dtype (B,Hkv,N,D). fa_p100_ext.cu:103-142."""
    return backward_into(q, k, v, dO, o, lse, causal, torch.float32)


def softmax_scale(head_dim):
    """The scale every kernel uses: 1/sqrt(D) (fa_p100_ext.cu:71, :117)."""
    return 1.0 / math.sqrt(head_dim)

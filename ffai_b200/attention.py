"""Python front end of libffai_attn.so over torch tensors.

Torch supplies device memory, streams and the process group; every
computation runs in the library's own CUDA kernels.  Each function builds a
descriptor (include/ffai_attn.h), calls the C ABI on the current torch
stream, and raises on errors.  A request the library does not serve raises
`Declined` (the C ABI's status 1).
"""

from __future__ import annotations

import ctypes
import threading

import torch

from . import _abi

_DT = {torch.float32: _abi.DT_F32, torch.bfloat16: _abi.DT_BF16, torch.float16: _abi.DT_F16}
_LAYOUT = {"heads": _abi.LAYOUT_HEADS_SPLIT, "token": _abi.LAYOUT_TOKEN_MAJOR, "kt": _abi.LAYOUT_KT}


class Declined(RuntimeError):
    """The library does not serve this shape/dtype (the reference's Ok(None))."""


class AttnError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"ffai_attn status {status}: {msg}")
        self.status = status


_ctx_lock = threading.Lock()
_contexts: dict[int, int] = {}


def context(device: int) -> int:
    """The library context of CUDA device `device` (created once, kept)."""
    with _ctx_lock:
        ctx = _contexts.get(device)
        if ctx is None:
            st = ctypes.c_int(0)
            ctx = _abi.load().ffai_attn_create(device, ctypes.byref(st))
            if not ctx:
                raise AttnError(st.value, _abi.last_error(None))
            _contexts[device] = ctx
        return ctx


def _check(status: int, ctx) -> None:
    if status == _abi.OK:
        return
    msg = _abi.last_error(ctx)
    if status == _abi.DECLINED:
        raise Declined(msg)
    raise AttnError(status, msg)


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(dev: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _need_cuda(*ts: torch.Tensor, strided: bool = False) -> torch.device:
    """The operands' common CUDA device; they must be contiguous unless
    `strided` (token-major views, checked by _operands)."""
    dev = ts[0].device
    for t in ts:
        if t.device.type != "cuda":
            raise ValueError("operands must be CUDA tensors")
        if t.device != dev:
            raise ValueError("operands must share one device")
        if not strided and not t.is_contiguous():
            raise ValueError("operands must be contiguous")
    return dev


def _dims(t: torch.Tensor, layout: str):
    """(B, H, N) of a q/k/v operand in the named layout."""
    if t.dim() != 4 or (t.shape[-1] != 64 and layout != "kt"):
        raise ValueError(f"expected a 4-d (..., 64) tensor, got {tuple(t.shape)}")
    if layout == "heads":
        return t.shape[0], t.shape[1], t.shape[2]
    if layout == "token":
        return t.shape[0], t.shape[2], t.shape[1]
    if layout == "kt":
        if t.shape[2] != 64:
            raise ValueError(f"K^T must be (B,H,64,N), got {tuple(t.shape)}")
        return t.shape[0], t.shape[1], t.shape[3]
    raise ValueError(layout)


def _token_stride(t: torch.Tensor):
    """Elements between tokens of a token-major (..., N, H, 64) view whose
    heads and head dims are dense (0 for a contiguous tensor), or None when
    the view has some other shape of strides."""
    if t.is_contiguous():
        return 0
    if t.stride(-1) != 1 or t.stride(-2) != 64:
        return None
    ts = t.stride(-3)
    if t.dim() == 4 and t.shape[0] > 1 and t.stride(0) != t.shape[1] * ts:
        return None
    return ts


def _operands(tensors, layouts):
    """Operands and their shared token stride: token-major views of one
    buffer with one stride (e.g. the three thirds of a fused QKV projection
    output) are passed as they are; anything else non-contiguous is copied."""
    strides = {_token_stride(t) for t, lay in zip(tensors, layouts) if lay == "token"}
    ts = 0
    if len(strides) == 1 and None not in strides:
        ts = strides.pop()
    for t, lay in zip(tensors, layouts):
        if not t.is_contiguous() and not (lay == "token" and ts):
            raise ValueError("operands must be contiguous, or token-major views with dense "
                             "heads and one shared token stride")
    return list(tensors), ts


def prefill(q, k, v, *, scale: float = 1.0, q_layout="heads", k_layout="heads",
            v_layout="heads", out_layout="heads", out_dtype=torch.float32, kv_len=None,
            with_lse=False, checked=False, causal=False, q_offset=0, out=None,
            inputs_stable=False):
    """softmax(scale q k^T) v over a batch of equal-length sequences.

    Layouts: "heads" (B,H,N,64), "token" (B,N,H,64) and, for k only, "kt"
    (B,H,64,N).  Returns out (and lse (B,H,Nq) or (H,B*Nq) when with_lse).
    `inputs_stable`: no work still pending on the stream writes q/k/v, so the
    kernel may read them while the preceding kernel finishes (back-to-back
    launches over independent batches overlap).
    """
    dev = _need_cuda(q, k, v, strided=True)
    B, H, Nq = _dims(q, q_layout)
    _, _, cap = _dims(k, k_layout)
    Nk = cap if kv_len is None else kv_len
    (q, k, v), ts = _operands((q, k, v), (q_layout, k_layout, v_layout))
    if out is None:
        shape = (B, H, Nq, 64) if out_layout == "heads" else (B, Nq, H, 64)
        out = torch.empty(shape, dtype=out_dtype, device=dev)
    lse = None
    if with_lse:
        lse = torch.empty((B, H, Nq) if out_layout == "heads" else (H, B * Nq),
                          dtype=torch.float32, device=dev)
    d = _abi.new_desc(batch=B, heads=H, q_len=Nq, kv_len=Nk, kv_capacity=cap,
                      q_dtype=_DT[q.dtype], kv_dtype=_DT[k.dtype], out_dtype=_DT[out.dtype],
                      q_layout=_LAYOUT[q_layout], k_layout=_LAYOUT[k_layout],
                      v_layout=_LAYOUT[v_layout], out_layout=_LAYOUT[out_layout],
                      causal=int(causal), q_offset=q_offset, scale=scale,
                      flags=(_abi.FLAG_CHECKED_F32 if checked else 0)
                      | (_abi.FLAG_INPUTS_STABLE if inputs_stable else 0), token_stride=ts)
    ctx = context(dev.index)
    st = _abi.load().ffai_attn_prefill(ctx, ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v), _ptr(out),
                                       _ptr(lse), _stream(dev))
    _check(st, ctx)
    return (out, lse) if with_lse else out


def decode(q, k, v, *, scale: float = 1.0, k_layout="heads", kv_len=None, out_dtype=torch.float32,
           with_lse=False, num_splits=0, causal=False, q_offset=0, out=None, kv_stable=False,
           kv_append_only=False, next_kv=None):
    """One decode step: q (B,H,1,64) against a K/V cache.

    k is (B,H,cap,64) ("heads") or (B,H,64,cap) ("kt"); v is (B,H,cap,64);
    `kv_len` <= cap keys are attended (default: all).  `kv_stable`: no work
    queued earlier on the stream writes k/v, so the kernel may start copying
    them before the preceding kernel finishes.  `kv_append_only`: that work
    writes at most the newest key (kv_len - 1), so the others may be copied
    early.  `next_kv`: (k, v) of the next decode call's cache (same shape and
    dtype), prefetched into L2 behind this call's own reads
    (ffai_attn_decode_prefetch; automatic split only).  Returns (B,H,1,64).
    """
    dev = _need_cuda(q, k, v)
    B, H, qlen = _dims(q, "heads")
    _, _, cap = _dims(k, k_layout)
    Nk = cap if kv_len is None else kv_len
    if out is None:
        out = torch.empty((B, H, 1, 64), dtype=out_dtype, device=dev)
    lse = torch.empty((B, H), dtype=torch.float32, device=dev) if with_lse else None
    d = _abi.new_desc(batch=B, heads=H, q_len=qlen, kv_len=Nk, kv_capacity=cap,
                      q_dtype=_DT[q.dtype], kv_dtype=_DT[k.dtype], out_dtype=_DT[out.dtype],
                      k_layout=_LAYOUT[k_layout], causal=int(causal), q_offset=q_offset,
                      scale=scale,
                      flags=(_abi.FLAG_KV_STABLE if kv_stable else 0)
                      | (_abi.FLAG_KV_APPEND_ONLY if kv_append_only else 0))
    ctx = context(dev.index)
    if next_kv is not None:
        nk, nv = next_kv
        if (nk.shape != k.shape or nv.shape != v.shape or nk.dtype != k.dtype
                or nv.dtype != v.dtype or nk.device != k.device or nv.device != v.device
                or not nk.is_contiguous() or not nv.is_contiguous()):
            raise ValueError("next_kv must match k and v in shape, dtype and device, contiguous")
        if num_splits != 0:
            raise ValueError("next_kv needs the automatic split (num_splits=0)")
        st = _abi.load().ffai_attn_decode_prefetch(ctx, ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v),
                                                   _ptr(nk), _ptr(nv), _ptr(out), _ptr(lse),
                                                   _stream(dev))
    else:
        st = _abi.load().ffai_attn_decode(ctx, ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v),
                                          _ptr(out), _ptr(lse), num_splits, _stream(dev))
    _check(st, ctx)
    return (out, lse) if with_lse else out


def decode_static(q, k, v, *, scale: float = 1.0, k_layout="heads", kv_len=None,
                  out_dtype=torch.float32, with_lse=False, num_splits=0, causal=False,
                  q_offset=0, out=None):
    """decode() through ffai_attn_decode_static: no context, no allocation by
    the library (its split scratch is a static device array), on q's device.
    Serialise calls on one device; see the header for the limits."""
    dev = _need_cuda(q, k, v)
    B, H, qlen = _dims(q, "heads")
    _, _, cap = _dims(k, k_layout)
    Nk = cap if kv_len is None else kv_len
    if out is None:
        out = torch.empty((B, H, 1, 64), dtype=out_dtype, device=dev)
    lse = torch.empty((B, H), dtype=torch.float32, device=dev) if with_lse else None
    d = _abi.new_desc(batch=B, heads=H, q_len=qlen, kv_len=Nk, kv_capacity=cap,
                      q_dtype=_DT[q.dtype], kv_dtype=_DT[k.dtype], out_dtype=_DT[out.dtype],
                      k_layout=_LAYOUT[k_layout], causal=int(causal), q_offset=q_offset,
                      scale=scale)
    with torch.cuda.device(dev):
        st = _abi.load().ffai_attn_decode_static(ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v),
                                                 _ptr(out), _ptr(lse), num_splits, _stream(dev))
    _check(st, None)
    return (out, lse) if with_lse else out


def varlen(q, k, v, cu_seqlens_q, cu_seqlens_k=None, *, scale: float = 1.0,
           out_dtype=torch.float32, with_lse=False, out=None, inputs_stable=False):
    """Ragged prefill over packed segments: q/k/v (T,H,64), host cu_seqlens.

    Segment s attends only within itself.  Returns out (T,H,64) [, lse (H,T)].
    `inputs_stable` as for prefill().
    """
    dev = _need_cuda(q, k, v, strided=True)
    if q.dim() != 3 or q.shape[-1] != 64:
        raise ValueError("varlen operands are (T, H, 64)")
    T, H = q.shape[0], q.shape[1]
    (q, k, v), ts = _operands((q, k, v), ("token", "token", "token"))
    cq = [int(x) for x in cu_seqlens_q]
    ck = cq if cu_seqlens_k is None else [int(x) for x in cu_seqlens_k]
    n_seg = len(cq) - 1
    arr_q = (ctypes.c_int32 * len(cq))(*cq)
    arr_k = (ctypes.c_int32 * len(ck))(*ck)
    if out is None:
        out = torch.empty((T, H, 64), dtype=out_dtype, device=dev)
    lse = torch.empty((H, T), dtype=torch.float32, device=dev) if with_lse else None
    d = _abi.new_desc(heads=H, q_dtype=_DT[q.dtype], kv_dtype=_DT[k.dtype],
                      out_dtype=_DT[out.dtype], q_layout=_abi.LAYOUT_TOKEN_MAJOR,
                      k_layout=_abi.LAYOUT_TOKEN_MAJOR, v_layout=_abi.LAYOUT_TOKEN_MAJOR,
                      out_layout=_abi.LAYOUT_TOKEN_MAJOR, scale=scale, token_stride=ts,
                      flags=_abi.FLAG_INPUTS_STABLE if inputs_stable else 0)
    ctx = context(dev.index)
    st = _abi.load().ffai_attn_varlen(ctx, ctypes.byref(d), arr_q, arr_k, n_seg, _ptr(q), _ptr(k),
                                      _ptr(v), _ptr(out), _ptr(lse), _stream(dev))
    _check(st, ctx)
    return (out, lse) if with_lse else out


def prefill_host(q, k, v, *, device: int = 0, scale: float = 1.0, out_dtype=torch.float32,
                 out=None, lse=None):
    """End-to-end prefill from HOST tensors (B,H,N,64): copies in, computes,
    copies out on the library's own streams, and returns the host output.
    Pinned (page-locked) host tensors overlap the copies with the kernels."""
    for t in (q, k, v):
        if t.device.type != "cpu" or not t.is_contiguous():
            raise ValueError("prefill_host takes contiguous host tensors")
    B, H, Nq = _dims(q, "heads")
    _, _, Nk = _dims(k, "heads")
    if out is None:
        out = torch.empty((B, H, Nq, 64), dtype=out_dtype, pin_memory=q.is_pinned())
    d = _abi.new_desc(batch=B, heads=H, q_len=Nq, kv_len=Nk, q_dtype=_DT[q.dtype],
                      kv_dtype=_DT[k.dtype], out_dtype=_DT[out.dtype], scale=scale)
    ctx = context(device)
    st = _abi.load().ffai_attn_prefill_host(ctx, ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v),
                                            _ptr(out), _ptr(lse))
    _check(st, ctx)
    return out


_worker_contexts: dict = {}


def worker_contexts(devices) -> list:
    """One library context per entry of `devices` (a device may repeat: each
    repetition gets a context of its own), created once and kept."""
    out, seen = [], {}
    with _ctx_lock:
        for dev in devices:
            slot = seen.get(dev, 0)
            seen[dev] = slot + 1
            ctx = _worker_contexts.get((dev, slot))
            if ctx is None:
                st = ctypes.c_int(0)
                ctx = _abi.load().ffai_attn_create(dev, ctypes.byref(st))
                if not ctx:
                    raise AttnError(st.value, _abi.last_error(None))
                _worker_contexts[(dev, slot)] = ctx
            out.append(ctx)
    return out


def multi_prefill_host(q, k, v, *, devices, scale: float = 1.0, out_dtype=torch.float32,
                       chunk_segments: int = 0, out=None, lse=None):
    """prefill_host over several devices: one worker thread per entry of
    `devices` takes chunks of `chunk_segments` sequences from a shared queue;
    a worker that fails hands its chunk back to the others.  Returns
    (out, failed_workers)."""
    for t in (q, k, v):
        if t.device.type != "cpu" or not t.is_contiguous():
            raise ValueError("multi_prefill_host takes contiguous host tensors")
    B, H, Nq = _dims(q, "heads")
    _, _, Nk = _dims(k, "heads")
    if out is None:
        out = torch.empty((B, H, Nq, 64), dtype=out_dtype, pin_memory=q.is_pinned())
    d = _abi.new_desc(batch=B, heads=H, q_len=Nq, kv_len=Nk, q_dtype=_DT[q.dtype],
                      kv_dtype=_DT[k.dtype], out_dtype=_DT[out.dtype], scale=scale)
    ctxs = worker_contexts(list(devices))
    arr = (ctypes.c_void_p * len(ctxs))(*ctxs)
    failed = ctypes.c_int32(0)
    st = _abi.load().ffai_attn_multi_prefill_host(arr, len(ctxs), ctypes.byref(d), _ptr(q), _ptr(k),
                                                  _ptr(v), _ptr(out), _ptr(lse), chunk_segments,
                                                  ctypes.byref(failed))
    _check(st, None)
    return out, failed.value


def profile(device: int = 0, enable: int = -1, read: bool = True):
    """Turn the context's launch timing on (1) / off (0) / leave it (-1);
    with `read`, return {op: (total ms, calls)} since the last read."""
    ctx = context(device)
    ms = (ctypes.c_double * 3)()
    n = (ctypes.c_int64 * 3)()
    st = _abi.load().ffai_attn_profile(ctx, enable, ms if read else None, n if read else None)
    _check(st, ctx)
    if not read:
        return None
    names = ("prefill", "decode", "varlen")
    return {names[i]: (ms[i], n[i]) for i in range(3)}


def sync(device: int | None = None) -> None:
    """Synchronise the current stream and raise if an in-kernel wait timed out."""
    dev = torch.cuda.current_device() if device is None else device
    ctx = context(dev)
    st = _abi.load().ffai_attn_sync(ctx, _stream(torch.device("cuda", dev)))
    _check(st, ctx)

"""The reference's custom-op surface, served by the B200 kernels.

Mirrors `crates/ffai-mercury/src/asr/flash_attn.rs` function for function:

    serves(kt, v) -> bool                       flash_attn.rs:104-129
    attend(q, kt, v, masked) -> Tensor | None   flash_attn.rs:218-264 ("flash-attn")
    attend_merged(q, kt, v) -> Tensor | None    flash_attn.rs:135-158 ("flash-attn-merged")

with the reference's argument meaning (q pre-scaled f32 (1,H,qlen,64), kt
(1,H,64,keys), v (1,H,keys,64)) and its decline contract: `None` means "shape
not served, take the three-op fallback", never an error.  Each call goes
through the C ABI (`ffai_flash_serves/attend/attend_merged`), the same entry
points a Rust crate binds.  Tensors live on a CUDA device here, where the
reference's lived on the CPU.
"""

from __future__ import annotations

import ctypes

import torch

from . import _abi
from .attention import AttnError, _DT, context

OP_NAME = "flash-attn"
MERGED_OP_NAME = "flash-attn-merged"


def _t4(t: torch.Tensor) -> _abi.Tensor4:
    x = _abi.Tensor4()
    x.data = t.data_ptr()
    dims = list(t.shape) + [0] * (4 - t.dim())
    for i in range(4):
        x.dims[i] = int(dims[i]) if i < t.dim() else 0
    x.dtype = _DT.get(t.dtype, -1)
    x.device = t.device.index if t.device.type == "cuda" else -1
    return x


def _stream(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def serves(kt: torch.Tensor, v: torch.Tensor) -> bool:
    """Whether the decode kernel will serve this K^T/V pair (cache-dtype choice)."""
    if kt.dim() != 4 or v.dim() != 4:
        return False
    return bool(_abi.load().ffai_flash_serves(ctypes.byref(_t4(kt)), ctypes.byref(_t4(v))))


def _run(fn, q, kt, v, out, *extra):
    if q.device.type != "cuda":
        return None  # host tensors: not served here (the reference declines off-CPU)
    for t in (q, kt, v):
        if t.dim() != 4 or not t.is_contiguous():
            return None
    ctx = context(q.device.index)
    st = fn(ctx, ctypes.byref(_t4(q)), ctypes.byref(_t4(kt)), ctypes.byref(_t4(v)), *extra,
            ctypes.byref(_t4(out)), _stream(q))
    if st == _abi.DECLINED:
        return None
    if st != _abi.OK:
        raise AttnError(st, _abi.last_error(ctx))
    return out


def attend(q: torch.Tensor, kt: torch.Tensor, v: torch.Tensor, masked: bool):
    """Fused attention (1,H,qlen,64), or None when this shape is not served."""
    if q.dim() != 4:
        return None
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    return _run(_abi.load().ffai_flash_attend, q, kt, v, out, ctypes.c_int32(int(masked)))


def attend_merged(q: torch.Tensor, kt: torch.Tensor, v: torch.Tensor):
    """Encoder attention returning (1, seq, heads*64) already merged, or None."""
    if q.dim() != 4:
        return None
    _, h, n, d = q.shape
    out = torch.empty((1, n, h * d), dtype=torch.float32, device=q.device)
    return _run(_abi.load().ffai_flash_attend_merged, q, kt, v, out)

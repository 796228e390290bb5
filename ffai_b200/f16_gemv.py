"""f16-weight GEMV on the device: the reference's F16Gemv
(crates/ffai-mercury/src/asr/f16_gemv.rs), the default path of the decoder's
single-row projections (QLinear::Half, text_decoder.rs:106-118, :231-252).

`F16Gemv.new(w, bias=None)` rounds a (rows, cols) weight matrix to f16 once,
or returns None for a shape the reference declines (cols not a multiple of
8); `forward(x)` maps (batch, cols) f32 activations (batch <= 8, e.g. the
beams of a step) to (batch, rows) f32 -- plus the bias, added after, as
QLinear::forward does -- in one pass over the weights, bit for bit what the
reference computes row by row.
"""

from __future__ import annotations

import ctypes

import torch

from . import _abi
from .attention import _DT, _check, _ptr, _stream, context

FLAG_WEIGHTS_STABLE = 0x2


def layout(rows: int, cols: int):
    """Bytes of the packed f16 weights, or None when the shape is not served."""
    n = ctypes.c_int64(0)
    st = _abi.load().ffai_f16_gemv_layout(rows, cols, ctypes.byref(n))
    return None if st != _abi.OK else n.value


class F16Gemv:
    def __init__(self, packed, rows: int, cols: int, bias=None):
        self.packed, self.rows, self.cols = packed, rows, cols
        self.bias = None if bias is None else bias.to(torch.float32).contiguous()
        self._written_by_previous = True

    @classmethod
    def new(cls, w: torch.Tensor, bias: torch.Tensor | None = None):
        if w.dim() != 2 or w.device.type != "cuda" or w.dtype not in _DT:
            return None
        rows, cols = w.shape
        nbytes = layout(rows, cols)
        if nbytes is None:
            return None
        w = w.contiguous()
        dev = w.device
        packed = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        ctx = context(dev.index)
        st = _abi.load().ffai_f16_gemv_pack(ctx, _ptr(w), _DT[w.dtype], rows, cols, _ptr(packed),
                                            _stream(dev))
        _check(st, ctx)
        return cls(packed, rows, cols, None if bias is None else bias.to(dev))

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if x.dtype != torch.float32:  # as cpu_fwd (f16_gemv.rs:146-149)
            raise TypeError("f16 GEMV: f32 activations only")
        if x.device != self.packed.device or x.shape[-1] != self.cols:
            raise ValueError(
                f"f16 GEMV: activations must be (batch, {self.cols}) on {self.packed.device}")
        x = x.reshape(-1, self.cols).contiguous()
        batch = x.shape[0]
        if out is None:
            out = torch.empty((batch, self.rows), dtype=torch.float32, device=x.device)
        elif out.shape != (batch, self.rows) or out.dtype != torch.float32 or not out.is_contiguous():
            raise ValueError(f"f16 GEMV: out must be contiguous f32 ({batch}, {self.rows})")
        flags = 0 if self._written_by_previous else FLAG_WEIGHTS_STABLE
        ctx = context(x.device.index)
        st = _abi.load().ffai_f16_gemv(ctx, _ptr(x), batch, _ptr(self.packed), _ptr(self.bias),
                                       self.rows, self.cols, _ptr(out), flags, _stream(x.device))
        _check(st, ctx)
        self._written_by_previous = False
        return out

    def unpacked(self, padded: bool = False) -> torch.Tensor:
        """The f16 weights (rows, cols) as the reference holds them (u16 bits)."""
        steps, R = (self.cols + 15) // 16, 8
        g = self.packed.numel() // (steps * R * 32)
        # [group][step][column c][row 0..7] -> (row, column)
        w = self.packed.view(torch.int16).view(g, steps, 16, R).permute(0, 3, 1, 2)
        w = w.reshape(g * R, steps * 16)[:, :self.cols]
        return w if padded else w[:self.rows]

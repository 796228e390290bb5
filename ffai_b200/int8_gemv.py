"""Block-scaled int8 GEMV on the device: the reference's Int8Vocab
(crates/ffai-mercury/src/asr/vocab_int8.rs) for the decoder's single-row
projections -- the vocabulary projection and the MLP layers that reuse it
(text_decoder.rs:94-104, :210-226, :945-969).

`Int8Gemv.new(w)` quantises a (rows, cols) weight matrix once, or returns
None for a shape it does not serve (as `Int8Vocab::new` does);
`forward(x)` maps (batch, cols) f32 activations (batch <= 8, e.g. the beams
of a step) to (batch, rows) f32 in one pass over the weights.  The quantised
weights live in the library's device layout of block records (weights and
scales of 16 rows x one block together); `unpacked()` returns them as the
reference holds them (row-major q, (rows, nblocks) scales, corr).
"""

from __future__ import annotations

import ctypes
import os

import torch

from . import _abi
from .attention import _DT, _check, _ptr, _stream, context

FLAG_WEIGHTS_STABLE = 0x2


def default_blk() -> int:
    """The reference's FFAI_VOCAB_BLK knob (knobs.rs:173): 32 unless set."""
    try:
        return int(os.environ.get("FFAI_VOCAB_BLK", "32"))
    except ValueError:
        return 32


def layout(rows: int, cols: int, blk: int):
    """(packed bytes, corr count) of the device layout, or None when the shape
    is not served."""
    n = [ctypes.c_int64(0) for _ in range(2)]
    st = _abi.load().ffai_int8_gemv_layout(rows, cols, blk, *(ctypes.byref(v) for v in n))
    return None if st != _abi.OK else tuple(v.value for v in n)


class Int8Gemv:
    def __init__(self, packed, corr, rows: int, cols: int, blk: int):
        self.packed, self.corr = packed, corr
        self.rows, self.cols, self.blk = rows, cols, blk
        # The first GEMV after the quantising kernel must not start streaming
        # the weights before that kernel ends; later ones may.
        self._written_by_previous = True

    @classmethod
    def new(cls, w: torch.Tensor, blk: int | None = None):
        """Quantise device weights w (rows, cols) of f32 / bf16 / f16."""
        blk = default_blk() if blk is None else blk
        if w.dim() != 2 or w.device.type != "cuda" or w.dtype not in _DT:
            return None
        rows, cols = w.shape
        sizes = layout(rows, cols, blk)
        if sizes is None:
            return None
        w = w.contiguous()
        dev = w.device
        packed = torch.empty(sizes[0], dtype=torch.uint8, device=dev)
        corr = torch.empty(sizes[1], dtype=torch.float32, device=dev)
        ctx = context(dev.index)
        st = _abi.load().ffai_int8_gemv_quantize(ctx, _ptr(w), _DT[w.dtype], rows, cols, blk,
                                                 _ptr(packed), _ptr(corr), _stream(dev))
        _check(st, ctx)
        return cls(packed, corr, rows, cols, blk)

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if x.dtype != torch.float32:  # as cpu_fwd (vocab_int8.rs:219-222)
            raise TypeError("int8 GEMV: f32 activations only")
        if x.device != self.packed.device or x.shape[-1] != self.cols:
            raise ValueError(
                f"int8 GEMV: activations must be (batch, {self.cols}) on {self.packed.device}")
        x = x.reshape(-1, self.cols).contiguous()
        if x.data_ptr() % 16:
            x = x.clone()  # the kernel reads the activations as 16-byte vectors
        batch = x.shape[0]
        if out is None:
            out = torch.empty((batch, self.rows), dtype=torch.float32, device=x.device)
        elif out.shape != (batch, self.rows) or out.dtype != torch.float32 or not out.is_contiguous():
            raise ValueError(f"int8 GEMV: out must be contiguous f32 ({batch}, {self.rows})")
        flags = 0 if self._written_by_previous else FLAG_WEIGHTS_STABLE
        ctx = context(x.device.index)
        st = _abi.load().ffai_int8_gemv(ctx, _ptr(x), batch, _ptr(self.packed), _ptr(self.corr),
                                        self.rows, self.cols, self.blk, _ptr(out), flags,
                                        _stream(x.device))
        _check(st, ctx)
        self._written_by_previous = False
        return out

    def unpacked(self, padded: bool = False):
        """(q (rows, cols) int8, scales (rows, cols / blk) f32, corr (rows,));
        with `padded`, the zero rows up to the group boundary too."""
        nb, blk, R = self.cols // self.blk, self.blk, 16
        g = self.corr.numel() // R
        recs = self.packed.view(g, nb, blk * R + 64)
        w = recs[:, :, :blk * R].reshape(g, nb, blk // 16, R, 16)  # (g, b, c, l, j)
        q = w.permute(0, 3, 1, 2, 4).reshape(g * R, self.cols).view(torch.int8)
        s = recs[:, :, blk * R:].contiguous().view(torch.float32).view(g, nb, R)
        # row l's scale sits at (l % 8) * 2 + l // 8
        perm = torch.tensor([(l % 8) * 2 + l // 8 for l in range(R)], device=s.device)
        s = s[:, :, perm].permute(0, 2, 1).reshape(g * R, nb)
        n = g * R if padded else self.rows
        return q[:n], s[:n], self.corr[:n]

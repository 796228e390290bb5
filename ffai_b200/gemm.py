"""bf16 GEMM with a fused epilogue on the tensor cores: the projections the
reference runs on candle's CPU GEMM around the attention -- the encoder MLP
(fc1 -> FastGelu -> fc2 + residual, audio_encoder.rs:147-165), the q/k/v
projection (whose (T, 3 * H * 64) output the attention reads in place as
three token-major views) and the out-projection.

    linear(a, w, bias=None, act=None, residual=None, out_dtype=torch.bfloat16)
        = act(a @ w.T + bias) + residual
"""

from __future__ import annotations

import torch

from . import _abi
from .attention import _check, _ptr, _stream, context

ACT = {None: 0, "fast_gelu": 1}
_OUT = {torch.float32: 0, torch.bfloat16: 1}


def linear(a: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
           act: str | None = None, residual: torch.Tensor | None = None,
           out_dtype: torch.dtype = torch.bfloat16, out: torch.Tensor | None = None) -> torch.Tensor:
    """a (M, K) bf16, w (N, K) bf16, bias (N) f32, residual (M, N) of out_dtype."""
    if a.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise TypeError("gemm: bf16 operands")
    if a.device.type != "cuda" or w.device != a.device:
        raise ValueError("gemm: operands on one CUDA device")
    if a.stride(-1) != 1 or w.stride(-1) != 1 or a.dim() != 2 or w.dim() != 2:
        raise ValueError("gemm: 2-d operands with unit column stride")
    M, K = a.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError("gemm: a (M, K) and w (N, K)")
    if bias is not None:
        bias = bias.to(device=a.device, dtype=torch.float32).contiguous()
    if residual is not None and (residual.dtype != out_dtype or residual.shape != (M, N)
                                 or residual.stride(-1) != 1):
        raise ValueError("gemm: residual (M, N) of the output dtype")
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    ctx = context(a.device.index)
    st = _abi.load().ffai_gemm_bf16(
        ctx, _ptr(a), a.stride(0), _ptr(w), w.stride(0), _ptr(bias), _ptr(residual),
        residual.stride(0) if residual is not None else 0, _ptr(out), out.stride(0), M, N, K,
        _OUT[out_dtype], ACT[act], _stream(a.device))
    _check(st, ctx)
    return out

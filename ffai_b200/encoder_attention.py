"""The encoder's self-attention block on B200: the caller side of the fused
attention, as code.

The reference's `EncoderAttention` (crates/ffai-mercury/src/asr/
text_decoder.rs:1010-1139) prepares the kernel's operands on the CPU: it
folds the whole 1/sqrt(head_dim) scale into the key weights at load
(`key_wt_scaled`, :1039-1051; Whisper's key projection has no bias), computes
q, v and the transposed k as three GEMMs (`ea_proj`, :1083-1096), splits the
heads and lays k out as K^T (`ea_prep`, :1099-1117), calls `attend_merged`
(:1121-1123) and applies the out-projection to the merged (1, seq, H*64)
result, one window at a time (:1069-1076).

Here the same block is three launches for a whole batch of windows:

  1. one fused q/k/v GEMM (`gemm.linear`) with the stacked weights
     [W_q; W_k / sqrt(head_dim); W_v] and biases [b_q; 0; b_v] -- the
     reference's scale fold, done once at load -- into a (T, 3 * H * 64) bf16
     buffer;
  2. the attention reading that buffer in place as three token-major views
     (`token_stride` = 3 * H * 64): no head split, no K transpose, scale 1;
  3. the out-projection GEMM on the attention's token-major (T, H * 64)
     output -- already the merged layout, so no head merge -- with the
     block's residual added in its epilogue when given.
"""

from __future__ import annotations

import torch

from . import attention
from .gemm import linear

HD = 64


def fold_qkv(wq: torch.Tensor, bq: torch.Tensor | None, wk: torch.Tensor, wv: torch.Tensor,
             bv: torch.Tensor | None):
    """Stacked q/k/v weights (3D, D) bf16 and biases (3D) f32 with the whole
    softmax scale folded into the key rows, as `key_wt_scaled` does
    (text_decoder.rs:1043-1046: (head_dim^-0.25)^2 on W_k).  For head_dim 64
    the factor is 1/8, a power of two, so the fold is exact in bf16."""
    D = wq.shape[1]
    if wq.shape != (D, D) or wk.shape != (D, D) or wv.shape != (D, D) or D % HD:
        raise ValueError("fold_qkv: square (D, D) projections with D a multiple of 64")
    scale = HD ** -0.5
    w = torch.cat([wq.float(), wk.float() * scale, wv.float()]).to(torch.bfloat16).contiguous()
    zeros = torch.zeros(D, device=wq.device)
    b = torch.cat([zeros if bq is None else bq.float(), zeros,
                   zeros if bv is None else bv.float()]).contiguous()
    return w, b


class EncoderAttention:
    """Whisper encoder self-attention (without the block's layer norm, which
    stays with the caller), weights as the checkpoint stores them: (out, in)
    projections, q and v with biases, k without, and the out-projection."""

    def __init__(self, wq, bq, wk, wv, bv, wo, bo, n_head: int):
        D = wq.shape[1]
        if D != n_head * HD:
            raise ValueError(f"EncoderAttention: d_model {D} != {n_head} heads x {HD}")
        self.n_head = n_head
        self.d_model = D
        self.w_qkv, self.b_qkv = fold_qkv(wq, bq, wk, wv, bv)
        self.w_o = wo.to(torch.bfloat16).contiguous()
        self.b_o = None if bo is None else bo.float().contiguous()

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None,
                out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """x (B, T, D) bf16 (the layer-normed input of B windows) -> (B, T, D)
        of out_dtype; with `residual` (B, T, D) of out_dtype, returns
        residual + attention(x), the block's residual stream."""
        B, T, D = x.shape
        if D != self.d_model or x.dtype != torch.bfloat16:
            raise ValueError("EncoderAttention.forward: x (B, T, d_model) bf16")
        H = self.n_head
        qkv = linear(x.reshape(B * T, D), self.w_qkv, self.b_qkv)  # (B*T, 3D) bf16
        views = [qkv[:, i * D:(i + 1) * D].view(B, T, H, HD) for i in range(3)]
        att = attention.prefill(*views, scale=1.0, q_layout="token", k_layout="token",
                                v_layout="token", out_layout="token",
                                out_dtype=torch.bfloat16)  # (B, T, H, 64): merged
        r = None if residual is None else residual.reshape(B * T, D)
        y = linear(att.view(B * T, D), self.w_o, self.b_o, residual=r, out_dtype=out_dtype)
        return y.view(B, T, D)

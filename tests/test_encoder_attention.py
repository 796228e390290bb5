"""The encoder self-attention block as the caller prepares it
(ffai_b200/encoder_attention.py; the reference's EncoderAttention,
text_decoder.rs:1010-1139): the scale fold, the fused q/k/v projection read
in place by the attention, and the out-projection on the merged output.

The attention stage is checked against the oracle (the reference's CPU
kernel) on exactly the bf16 q/k/v the projection produced, at the bf16 bar;
the whole block against an fp32 restatement of the reference's arithmetic on
the same bf16 weights and input.  The block rounds to bf16 at three points
(the q/k/v projection's output, the attention's output, and the operands of
both GEMMs), so its bar is relative to the output's scale: max |err| <= 2e-2
and mean |err| <= 2e-3 of max |ref|."""

import numpy as np
import pytest
import torch

from helpers import assert_bf16_close, f32np

DEV = "cuda:0"
BLOCK_MAX_REL = 2e-2
BLOCK_MEAN_REL = 2e-3


def _weights(D, seed):
    g = torch.Generator().manual_seed(seed)
    s = D ** -0.5
    wq, wk, wv, wo = (torch.randn(D, D, generator=g) * s for _ in range(4))
    bq, bv, bo = (torch.randn(D, generator=g) * 0.1 for _ in range(3))
    return wq, bq, wk, wv, bv, wo, bo


def test_fold_qkv_scales_the_key_rows_exactly():
    from ffai_b200.encoder_attention import fold_qkv
    D = 128
    wq, bq, wk, wv, bv, _, _ = _weights(D, 1)
    w, b = fold_qkv(wq, bq, wk, wv, bv)
    assert w.shape == (3 * D, D) and w.dtype == torch.bfloat16
    # 1/8 is a power of two: folding it into the bf16 key weights is exact
    assert torch.equal(w[D:2 * D], (wk.to(torch.bfloat16).float() / 8).to(torch.bfloat16))
    assert torch.equal(w[:D], wq.to(torch.bfloat16))
    assert torch.equal(w[2 * D:], wv.to(torch.bfloat16))
    assert torch.equal(b[D:2 * D], torch.zeros(D))  # Whisper's key projection has no bias
    assert torch.equal(b[:D], bq) and torch.equal(b[2 * D:], bv)
    with pytest.raises(ValueError):
        fold_qkv(wq[:, :100], bq, wk, wv, bv)


def _reference_block(x, wq, bq, wk, wv, bv, wo, bo, H):
    """The reference's encoder attention in fp32 on the bf16-rounded weights
    and input: q = x Wq^T + bq, k^T = (Wk / 8) x^T, v = x Wv^T + bv,
    softmax(q k) v per head, merged, then the out-projection."""
    r = lambda t: t.to(torch.bfloat16).float()
    x, wq, wk, wv, wo = r(x), r(wq), r(wk), r(wv), r(wo)
    B, T, D = x.shape
    q = (x @ wq.T + bq).view(B, T, H, 64).transpose(1, 2)
    k = (x @ (wk / 8).T).view(B, T, H, 64).transpose(1, 2)
    v = (x @ wv.T + bv).view(B, T, H, 64).transpose(1, 2)
    att = torch.softmax(q @ k.transpose(-1, -2), -1) @ v
    return att.transpose(1, 2).reshape(B, T, D) @ wo.T + bo


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,H", [(2, 1500, 6), (1, 300, 8), (3, 257, 6)])
def test_encoder_block_matches_reference(oracle, B, T, H):
    from ffai_b200 import attention
    from ffai_b200.encoder_attention import EncoderAttention
    from ffai_b200.gemm import linear
    D = H * 64
    ws = _weights(D, 3)
    blk = EncoderAttention(*(t.to(DEV) for t in ws), n_head=H)
    g = torch.Generator().manual_seed(11)
    x = torch.randn(B, T, D, generator=g).to(torch.bfloat16)
    y = blk.forward(x.to(DEV))
    attention.sync(0)

    # the attention stage on the projection's own bf16 output, against the
    # reference's kernel (q pre-scaled by the fold, K^T as the reference lays it)
    qkv = linear(x.to(DEV).reshape(B * T, D), blk.w_qkv, blk.b_qkv)
    q, k, v = (f32np(qkv[:, i * D:(i + 1) * D]).reshape(B, T, H, 64).transpose(0, 2, 1, 3)
               for i in range(3))
    U = B * H
    want_att = oracle.flash_units(np.ascontiguousarray(q.reshape(U, T, 64)),
                                  np.ascontiguousarray(np.swapaxes(k.reshape(U, T, 64), 1, 2)),
                                  np.ascontiguousarray(v.reshape(U, T, 64)))
    views = [qkv[:, i * D:(i + 1) * D].view(B, T, H, 64) for i in range(3)]
    att = attention.prefill(*views, scale=1.0, q_layout="token", k_layout="token",
                            v_layout="token", out_layout="token")
    got_att = f32np(att).transpose(0, 2, 1, 3).reshape(U, T, 64)
    assert_bf16_close(got_att, want_att, "attention on the fused projection's views")

    # the whole block against fp32
    ref = _reference_block(x, *ws, H).numpy()
    err = np.abs(f32np(y) - ref)
    scale = np.abs(ref).max()
    assert err.max() <= BLOCK_MAX_REL * scale, (err.max(), scale)
    assert err.mean() <= BLOCK_MEAN_REL * scale, (err.mean(), scale)


@pytest.mark.gpu
def test_encoder_block_residual_in_the_epilogue():
    from ffai_b200.encoder_attention import EncoderAttention
    B, T, H = 2, 300, 6
    D = H * 64
    blk = EncoderAttention(*(t.to(DEV) for t in _weights(D, 5)), n_head=H)
    g = torch.Generator(device=DEV).manual_seed(2)
    x = torch.randn(B, T, D, device=DEV, generator=g).to(torch.bfloat16)
    res = torch.randn(B, T, D, device=DEV, generator=g)
    y = blk.forward(x)
    yr = blk.forward(x, residual=res)
    # the epilogue adds the residual to the f32 result: one f32 rounding
    assert torch.allclose(yr, y + res, rtol=0, atol=1e-5 * (1 + res.abs().max().item()))
    with pytest.raises(ValueError):
        blk.forward(x.float())

"""The reference's own tests for this path (flash_attn.rs:1000-1040), run
against the B200 library through its mirrored surface: serves / attend /
attend_merged with the reference's shapes, f32 operands and decline rules."""

import numpy as np
import pytest
import torch

from ffai_b200 import flash_attn
from helpers import assert_bf16_close, f32np

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
HD = 64


def _randn(g, *shape, scale=1.0):
    return torch.randn(*shape, generator=g) * scale


def test_matches_three_op_path(oracle, monkeypatch):
    """flash_attn.rs:1005-1021 with its exact bar, max |delta| < 1e-4, in the
    checked f32 mode (the bf16 tensor-core path is held to the bf16 bar below)."""
    monkeypatch.setenv("FFAI_ATTN_CHECKED_F32", "1")
    g = torch.Generator().manual_seed(0)
    h, seq = 4, 512
    q = _randn(g, 1, h, seq, HD)
    k = _randn(g, 1, h, HD, seq)
    v = _randn(g, 1, h, seq, HD)
    ours = flash_attn.attend(q.to(DEV), k.to(DEV), v.to(DEV), False)
    assert ours is not None
    want = oracle.three_op(q.numpy(), k.numpy(), v.numpy())
    d = np.abs(f32np(ours) - want).max()
    assert d < 1e-4, f"max |delta| {d:e} exceeds tolerance"


def test_attend_bf16_path_vs_oracle(oracle, monkeypatch):
    """Default (tensor-core) path on the reference's encoder shape, against
    the oracle on the same bf16-rounded operands."""
    monkeypatch.delenv("FFAI_ATTN_CHECKED_F32", raising=False)
    g = torch.Generator().manual_seed(1)
    h, seq = 6, 1500
    q = _randn(g, 1, h, seq, HD, scale=0.5 / 8)  # pre-scaled, as callers pass it
    k = _randn(g, 1, h, HD, seq, scale=0.5)
    v = _randn(g, 1, h, seq, HD)
    ours = flash_attn.attend(q.to(DEV), k.to(DEV), v.to(DEV), False)
    rb = [t.to(torch.bfloat16).float().numpy() for t in (q, k, v)]
    want = oracle.attend(*rb, False)
    assert_bf16_close(f32np(ours), want, "attend bf16")
    merged = flash_attn.attend_merged(q.to(DEV), k.to(DEV), v.to(DEV))
    assert merged.shape == (1, seq, h * HD)
    assert torch.equal(merged[0].view(seq, h, HD).transpose(0, 1), ours[0])


def test_declines_unsupported_shapes():
    """flash_attn.rs:1024-1039."""
    g = torch.Generator().manual_seed(2)
    q = _randn(g, 1, 4, 1, HD).to(DEV)
    k = _randn(g, 1, 4, HD, 1).to(DEV)
    v = _randn(g, 1, 4, 1, HD).to(DEV)
    assert flash_attn.attend(q, k, v, False) is None
    q = _randn(g, 1, 4, 512, HD).to(DEV)
    k = _randn(g, 1, 4, HD, 512).to(DEV)
    v = _randn(g, 1, 4, 512, HD).to(DEV)
    assert flash_attn.attend(q, k, v, True) is None
    # host tensors are not served by a GPU library
    assert flash_attn.attend(q.cpu(), k.cpu(), v.cpu(), False) is None
    # below the encoder floor, and q_len neither 1 nor keys
    assert flash_attn.attend_merged(q[:, :, :255].contiguous(), k[..., :255].contiguous(),
                                    v[:, :, :255].contiguous()) is None
    assert flash_attn.attend(q[:, :, :300].contiguous(), k, v, False) is None


def test_decode_through_surface_f16_cache(oracle):
    """Cross-attention as the reference stores it: f16 K^T/V cache, f32 q."""
    g = torch.Generator().manual_seed(3)
    h, keys = 12, 1500
    q = _randn(g, 1, h, 1, HD, scale=0.5)
    kt = _randn(g, 1, h, HD, keys).to(torch.float16)
    v = _randn(g, 1, h, keys, HD).to(torch.float16)
    assert flash_attn.serves(kt.to(DEV), v.to(DEV))
    ours = flash_attn.attend(q.to(DEV), kt.to(DEV), v.to(DEV), False)
    want = oracle.attend_f16kv(q.numpy(), kt.numpy().view(np.uint16), v.numpy().view(np.uint16))
    d = np.abs(f32np(ours) - want).max()
    assert d < 1e-5, f"max |delta| {d:e}"


def test_decode_through_surface_f32_self_attention(oracle):
    g = torch.Generator().manual_seed(4)
    h = 12
    for keys in (8, 33, 448):
        q = _randn(g, 1, h, 1, HD, scale=0.5)
        kt = _randn(g, 1, h, HD, keys)
        v = _randn(g, 1, h, keys, HD)
        ours = flash_attn.attend(q.to(DEV), kt.to(DEV), v.to(DEV), False)
        want = oracle.attend(q.numpy(), kt.numpy(), v.numpy(), False)
        assert np.abs(f32np(ours) - want).max() < 1e-5
    # 7 keys: below FFAI_DECODE_MIN_KEYS, declined like the reference
    kt = _randn(g, 1, h, HD, 7).to(DEV)
    v = _randn(g, 1, h, 7, HD).to(DEV)
    assert flash_attn.attend(q.to(DEV), kt, v, False) is None


def test_serves_matches_reference_predicate(oracle):
    for keys, heads_v in [(1500, 6), (256, 6), (255, 6), (1500, 5)]:
        kt = torch.empty(1, 6, HD, keys, device=DEV)
        v = torch.empty(1, heads_v, keys, HD, device=DEV)
        assert flash_attn.serves(kt, v) == oracle.serves(kt.shape, v.shape)


def test_profile_counts_calls():
    """Opt-in launch timing: CUDA events per call, read and reset."""
    from ffai_b200 import attention, workloads
    attention.profile(0, enable=1)  # on; also clears earlier records
    q, k, v = workloads.decode_inputs(448, seed=30, device="cuda")
    for _ in range(3):
        attention.decode(q, k, v)
    g = torch.Generator().manual_seed(1)
    x = (torch.randn(1, 2, 256, 64, generator=g) * 0.5).to(torch.bfloat16).cuda()
    attention.prefill(x, x, x, scale=0.125)
    stats = attention.profile(0, enable=0)
    assert stats["decode"][1] == 3 and stats["decode"][0] > 0
    assert stats["prefill"][1] == 1 and stats["prefill"][0] > 0
    assert attention.profile(0)["decode"] == (0.0, 0)

"""bf16 GEMM with the fused epilogue (bias, the reference's FastGelu,
residual): against a plain PyTorch fp32 reference on the same bf16-rounded
operands (f32 accumulation in a different order: relative tolerance 2e-5 of
the row's magnitude for f32 output, one bf16 ulp for bf16 output), and the
activation bit for bit against the oracle's restatement of gelu_scalar
(text_decoder.rs:341-350)."""

import numpy as np
import pytest
import torch

DEV = "cuda:0"


def test_oracle_fast_gelu_tracks_tanh_gelu(oracle):
    # the reference measured max |error| 1.8e-4 against the tanh form
    x = np.linspace(-8, 8, 4001, dtype=np.float32)
    want = 0.5 * x * (1 + np.tanh(np.sqrt(2 / np.pi) * (x + 0.044715 * x.astype(np.float64) ** 3)))
    assert np.abs(oracle.fast_gelu(x) - want).max() < 2e-4


def test_abi_declares_gemm():
    from ffai_b200 import _abi
    assert hasattr(_abi.load(), "ffai_gemm_bf16")


def _ref(a, w, bias, act, residual, oracle):
    y = a.float() @ w.float().T
    if bias is not None:
        y = y + bias.float()
    if act == "fast_gelu":
        y = torch.from_numpy(oracle.fast_gelu(y.cpu().numpy())).to(y.device)
    if residual is not None:
        y = y + residual.float()
    return y


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [
    (1500, 5120, 1280), (1500, 1280, 5120), (3000, 3840, 1280), (1500, 1280, 1280),
    (200, 384, 384), (129, 288, 72), (1, 32, 8),
])
@pytest.mark.parametrize("variant", ["plain", "bias_gelu", "bias_residual", "bias_gelu_residual"])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_gemm_matches_fp32_reference(oracle, M, N, K, variant, out_dtype):
    from ffai_b200.gemm import linear
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    a = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=DEV, generator=g) / K ** 0.5).to(torch.bfloat16)
    bias = torch.randn(N, device=DEV, generator=g) if variant != "plain" else None
    act = "fast_gelu" if "gelu" in variant else None
    res = torch.randn(M, N, device=DEV, generator=g).to(out_dtype) if "residual" in variant else None
    got = linear(a, w, bias, act, res, out_dtype=out_dtype)
    torch.cuda.synchronize()
    want = _ref(a, w, bias, act, res, oracle)
    scale = want.abs().amax(dim=1, keepdim=True).clamp_min(1e-3)
    err = ((got.float() - want).abs() / scale).max().item()
    tol = 2e-5 if out_dtype == torch.float32 else 2 ** -8
    assert err <= tol, f"max relative error {err:.3e}"


def _assert_bits_equal(got, want, x):
    """Bit-for-bit, NaN where the reference gives NaN; names the first misses."""
    nan = np.isnan(want)
    bad = (np.isnan(got) != nan) | (~nan & (got.view(np.int32) != want.view(np.int32)))
    idx = np.argwhere(bad)[:8]
    assert not bad.any(), (f"{int(bad.sum())} mismatches, first: "
                           + ", ".join(f"t={x[tuple(i)]!r} got={got[tuple(i)]!r} "
                                       f"want={want[tuple(i)]!r}" for i in idx))


@pytest.mark.gpu
def test_gemm_epilogue_fast_gelu_bit_exact(oracle):
    # a[m][0] = t_m, b[n][0] = 1: the accumulator is t_m exactly; bias b_n
    # moves it off the bf16 grid (the same f32 add on both sides)
    from ffai_b200.gemm import linear
    M, N, K = 257, 64, 8
    t = torch.linspace(-7, 7, M).to(torch.bfloat16)
    a = torch.zeros(M, K, dtype=torch.bfloat16)
    a[:, 0] = t
    w = torch.zeros(N, K, dtype=torch.bfloat16)
    w[:, 0] = 1
    bias = torch.linspace(-0.37, 0.41, N, dtype=torch.float32)
    got = linear(a.to(DEV), w.to(DEV), bias.to(DEV), "fast_gelu", out_dtype=torch.float32)
    x = (t.float()[:, None] + bias[None, :]).numpy().astype(np.float32)
    want = oracle.fast_gelu(x)
    _assert_bits_equal(got.cpu().numpy(), want, x)


@pytest.mark.gpu
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_gemm_epilogue_fast_gelu_bit_exact_wide(oracle, out_dtype):
    # ~1M pre-activations t_m + b_n spread over every binade from 1e-30 to
    # 1e12 of both signs (plus +-inf and zero), through the epilogue's
    # division-free rounding of num / den: bit for bit, NaN where the
    # reference gives NaN; f32 output (8 epilogue warps) and bf16 output
    # (12 epilogue warps, the value rounded to nearest even)
    from ffai_b200.gemm import linear
    M, N, K = 256, 4096, 8
    g = np.random.default_rng(11)
    t = torch.from_numpy(np.concatenate([np.linspace(-6, 6, M - 16), np.zeros(16)])
                         .astype(np.float32)).to(torch.bfloat16)
    a = torch.zeros(M, K, dtype=torch.bfloat16)
    a[:, 0] = t
    w = torch.zeros(N, K, dtype=torch.bfloat16)
    w[:, 0] = 1
    mag = 10.0 ** g.uniform(-30, 12, N)
    bias = (mag * g.choice([-1.0, 1.0], N)).astype(np.float32)
    bias[:4] = [np.inf, -np.inf, 0.0, -0.0]
    bias[4:1024] = g.uniform(-8, 8, 1020).astype(np.float32)  # the rational's own range
    got = linear(a.to(DEV), w.to(DEV), torch.from_numpy(bias).to(DEV), "fast_gelu",
                 out_dtype=out_dtype).float().cpu().numpy()
    x = (t.float()[:, None] + torch.from_numpy(bias)[None, :]).numpy().astype(np.float32)
    want = oracle.fast_gelu(x)
    if out_dtype == torch.bfloat16:  # the bf16 store rounds to nearest even
        want = torch.from_numpy(want).to(torch.bfloat16).float().numpy()
    _assert_bits_equal(got, want, x)


@pytest.mark.gpu
def test_gemm_qkv_feeds_attention_in_place():
    # the fused q/k/v projection's output read by the prefill as token-major views
    from ffai_b200 import attention
    from ffai_b200.gemm import linear
    T, H, D = 300, 6, 64
    g = torch.Generator(device=DEV).manual_seed(7)
    x = torch.randn(T, H * D, device=DEV, generator=g).to(torch.bfloat16)
    wqkv = (torch.randn(3 * H * D, H * D, device=DEV, generator=g) / (H * D) ** 0.5).to(torch.bfloat16)
    qkv = linear(x, wqkv)  # (T, 3 H D) bf16
    q, k, v = (qkv[:, i * H * D:(i + 1) * H * D].view(1, T, H, D) for i in range(3))
    out = attention.prefill(q, k, v, scale=D ** -0.5, q_layout="token", k_layout="token",
                            v_layout="token")  # (1, H, T, 64)
    qr, kr, vr = (t.float().permute(0, 2, 1, 3) for t in (q, k, v))
    want = torch.softmax(qr @ kr.transpose(-1, -2) * D ** -0.5, -1) @ vr
    err = (out.float() - want).abs().max().item()
    assert err < 2e-2


@pytest.mark.gpu
def test_gemm_rejects_bad_shapes():
    from ffai_b200 import attention
    from ffai_b200.gemm import linear
    a = torch.randn(16, 64, device=DEV).to(torch.bfloat16)
    with pytest.raises(attention.Declined):
        linear(a, torch.randn(40, 64, device=DEV).to(torch.bfloat16))  # N % 32
    with pytest.raises(TypeError):
        linear(a.float(), torch.randn(32, 64, device=DEV))

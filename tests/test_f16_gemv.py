"""f16-weight GEMV: the reference's F16Gemv (f16_gemv.rs).

CPU: the oracle (oracle/f16_gemv_ref.cpp) against the reference's own tests
(f16_gemv.rs:201-247) and against an exact restatement (rational arithmetic,
one rounding per fused multiply-add); the C ABI's layout sizes.  GPU: packing
and GEMV through the C ABI equal the oracle bit for bit (NaN payloads aside)
for the decoder's shapes, the 8-column tail, every batch 1..8, with and
without bias, and non-finite inputs.
"""

from fractions import Fraction

import numpy as np
import pytest
import torch

DEV = "cuda:0"


def _round_f32(v: Fraction) -> np.float32:
    """Nearest-even f32 of an exact rational (finite, normal range)."""
    if v == 0:
        return np.float32(0.0)
    sign = -1 if v < 0 else 1
    a = abs(v)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    while Fraction(2) ** e > a:
        e -= 1
    while Fraction(2) ** (e + 1) <= a:
        e += 1
    scale = Fraction(2) ** (e - 23)  # 24-bit significand
    m = a / scale
    q, r = divmod(m.numerator, m.denominator)
    rem = Fraction(r, m.denominator)
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and q % 2 == 1):
        q += 1
    return np.float32(sign * float(q * scale))


def _fma(a, b, c):
    return _round_f32(Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c)))


def _exact_dot(w16, x):
    """dot_f16 (f16_gemv.rs:170-194) in exact arithmetic, rounding per fma."""
    w = w16.view(np.float16).astype(np.float32)
    d = len(x)
    acc0, acc1 = [np.float32(0)] * 8, [np.float32(0)] * 8
    k = 0
    while k + 16 <= d:
        acc0 = [_fma(w[k + i], x[k + i], acc0[i]) for i in range(8)]
        acc1 = [_fma(w[k + 8 + i], x[k + 8 + i], acc1[i]) for i in range(8)]
        k += 16
    while k + 8 <= d:
        acc0 = [_fma(w[k + i], x[k + i], acc0[i]) for i in range(8)]
        k += 8
    a = [np.float32(acc0[i] + acc1[i]) for i in range(8)]
    s = [np.float32(a[i] + a[i + 4]) for i in range(4)]
    return np.float32(np.float32(s[0] + s[2]) + np.float32(s[1] + s[3]))


def _same(a, b):
    a, b = np.ascontiguousarray(a, np.float32), np.ascontiguousarray(b, np.float32)
    na, nb = np.isnan(a), np.isnan(b)
    return np.array_equal(na, nb) and np.array_equal(a.view(np.int32)[~na], b.view(np.int32)[~nb])


def test_oracle_matches_f32_matmul(oracle):
    # restates f16_gemv.rs:205-229 with seeded inputs
    rng = np.random.default_rng(3)
    w = rng.standard_normal((1536, 384), dtype=np.float32)
    x = rng.standard_normal((1, 384), dtype=np.float32)
    ours = oracle.f16_gemv(x, oracle.f16_weights(w))[0]
    want = (x @ w.T)[0]
    assert np.abs(ours - want).max() / np.abs(want).max() < 5e-3


def test_oracle_declines_shapes_it_cannot_serve(oracle):
    # f16_gemv.rs:231-237
    assert oracle.f16_weights(np.ones((16, 12), np.float32)) is None


@pytest.mark.parametrize("cols", [8, 24, 32, 40])
def test_oracle_matches_exact_restatement(oracle, cols):
    rng = np.random.default_rng(cols)
    w = rng.standard_normal((3, cols), dtype=np.float32)
    x = rng.standard_normal((2, cols), dtype=np.float32) * np.float32(3)
    bias = rng.standard_normal(3, dtype=np.float32)
    w16 = oracle.f16_weights(w)
    got = oracle.f16_gemv(x, w16, bias, threads=1)
    for b in range(2):
        for r in range(3):
            want = np.float32(_exact_dot(w16[r], x[b]) + bias[r])
            assert got[b, r].view(np.int32) == want.view(np.int32), (b, r)


def test_abi_layout():
    from ffai_b200.f16_gemv import layout
    assert layout(1280, 1280) == 160 * 80 * 256
    assert layout(3, 8) == 1 * 1 * 256
    assert layout(7, 1288) == 1 * 81 * 256
    assert layout(9, 16) == 2 * 1 * 256
    for rows, cols in [(16, 12), (0, 16), (4, 0), (4, 65544)]:
        assert layout(rows, cols) is None


# --------------------------------------------------------------------------- GPU


def _weights(rows, cols, seed):
    rng = np.random.default_rng(seed)
    return rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.05)


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols,dtype", [
    (1280, 1280, torch.float32), (5120, 1280, torch.bfloat16), (1280, 5120, torch.float16),
    (7, 1288, torch.float32), (3, 8, torch.float32),
])
def test_pack_matches_oracle(oracle, rows, cols, dtype):
    from ffai_b200.f16_gemv import F16Gemv
    w = torch.from_numpy(_weights(rows, cols, rows + cols)).to(dtype)
    q = F16Gemv.new(w.to(DEV))
    torch.cuda.synchronize()
    want = oracle.f16_weights(w.float().numpy())
    assert np.array_equal(q.unpacked().cpu().numpy().view(np.uint16), want)
    pad = q.unpacked(padded=True)
    assert not pad[rows:].any()


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", [
    (1280, 1280), (5120, 1280), (1280, 5120), (1536, 384), (3840, 1280), (7, 1288), (3, 8),
    (51865, 384), (33, 24),
])
@pytest.mark.parametrize("batch", [1, 2, 5, 8])
@pytest.mark.parametrize("with_bias", [False, True])
def test_gemv_matches_oracle(oracle, rows, cols, batch, with_bias):
    from ffai_b200.f16_gemv import F16Gemv
    w = _weights(rows, cols, 5 * rows + cols)
    rng = np.random.default_rng(rows + batch)
    x = rng.standard_normal((batch, cols), dtype=np.float32)
    bias = rng.standard_normal(rows, dtype=np.float32) if with_bias else None
    q = F16Gemv.new(torch.from_numpy(w).to(DEV),
                    None if bias is None else torch.from_numpy(bias).to(DEV))
    xd = torch.from_numpy(x).to(DEV)
    out = q.forward(xd)
    out2 = q.forward(xd)  # weights stable: streamed ahead of the preceding kernel's end
    torch.cuda.synchronize()
    assert torch.equal(out, out2)
    want = oracle.f16_gemv(x, oracle.f16_weights(w), bias)
    got = out.cpu().numpy()
    assert _same(got, want), f"max |diff| {np.nanmax(np.abs(got - want))}"


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols,batch", [(1280, 5120, 5), (3840, 1280, 1), (33, 24, 3)])
def test_gemv_unaligned_activations(oracle, rows, cols, batch):
    # activations 4 bytes past a 16-byte boundary: staged with 4-byte loads
    from ffai_b200.f16_gemv import F16Gemv
    w = _weights(rows, cols, rows * cols + 3)
    rng = np.random.default_rng(cols + batch)
    x = rng.standard_normal((batch, cols), dtype=np.float32)
    q = F16Gemv.new(torch.from_numpy(w).to(DEV))
    buf = torch.empty(batch * cols + 1, device=DEV)
    xd = buf[1:].view(batch, cols)
    xd.copy_(torch.from_numpy(x))
    assert xd.data_ptr() % 16 == 4
    got = q.forward(xd).cpu().numpy()
    assert _same(got, oracle.f16_gemv(x, oracle.f16_weights(w)))


@pytest.mark.gpu
def test_gemv_nonfinite_inputs(oracle):
    from ffai_b200.f16_gemv import F16Gemv
    w = _weights(6, 40, 1)
    w[1, 3] = 1e6          # beyond f16: inf
    w[2, 17] = np.nan
    x = np.random.default_rng(2).standard_normal((3, 40), dtype=np.float32)
    x[1, 5] = np.inf
    x[2, 33] = np.nan
    q = F16Gemv.new(torch.from_numpy(w).to(DEV))
    got = q.forward(torch.from_numpy(x).to(DEV)).cpu().numpy()
    assert _same(got, oracle.f16_gemv(x, oracle.f16_weights(w)))


@pytest.mark.gpu
def test_gemv_declines_and_rejects():
    from ffai_b200 import _abi, attention
    from ffai_b200.f16_gemv import F16Gemv
    assert F16Gemv.new(torch.randn(16, 12, device=DEV)) is None
    assert F16Gemv.new(torch.randn(16, 16)) is None  # host tensor: not served here
    q = F16Gemv.new(torch.randn(64, 64, device=DEV))
    with pytest.raises(attention.AttnError) as e:
        q.forward(torch.randn(9, 64, device=DEV))
    assert e.value.status == _abi.ERR_INVALID
    with pytest.raises(TypeError):
        q.forward(torch.randn(1, 64, device=DEV, dtype=torch.float16))

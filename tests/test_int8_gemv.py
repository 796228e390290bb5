"""Int8 block-scaled GEMV: the reference's Int8Vocab (vocab_int8.rs).

CPU: the oracle (oracle/vocab_int8_ref.cpp) against the reference's own
tests (vocab_int8.rs:401-438) and against a scalar numpy restatement; the
C ABI's scale pitch.  GPU: quantisation and GEMV through the C ABI equal the
oracle bit for bit, including rounding ties, zero blocks, zero activation
rows, ragged row counts and every block width the reference serves.
"""

import numpy as np
import pytest
import torch

from ffai_b200 import _abi

DEV = "cuda:0"


def _round_half_away(x):
    t = np.trunc(x)
    return t + np.where(np.abs(x - t) >= np.float32(0.5), np.sign(x), np.float32(0)).astype(np.float32)


def _clamp_cast(r, lo, hi):
    """f32::clamp then Rust's saturating `as` cast: NaN -> 0."""
    with np.errstate(invalid="ignore"):
        return np.where(np.isnan(r), 0, np.clip(np.nan_to_num(r, nan=0.0), lo, hi)).astype(np.int64)


def _scalar_reference(w, x, blk):
    """Int8Vocab::new + cpu_fwd + dot_i8_blocked with numpy f32 scalars."""
    with np.errstate(all="ignore"):  # inf * 0 and inf / inf are part of the non-finite cases
        return _scalar_reference_steps(w, x, blk)


def _scalar_reference_steps(w, x, blk):
    f = np.float32
    vocab, d = w.shape
    nb = d // blk
    out = np.empty((x.shape[0], vocab), np.float32)
    q = np.empty((vocab, d), np.int64)
    bs = np.empty((vocab, nb), np.float32)
    corr = np.empty(vocab, np.float32)
    for v in range(vocab):
        c = f(0)
        for b in range(nb):
            bw = w[v, b * blk:(b + 1) * blk]
            amax = f(np.nanmax(np.concatenate([[0], np.abs(bw)])))
            sc = amax / f(127) if amax > 0 else f(1)
            bs[v, b] = sc
            with np.errstate(invalid="ignore", divide="ignore"):
                qb = _clamp_cast(_round_half_away(bw / sc), -127, 127)
            q[v, b * blk:(b + 1) * blk] = qb
            c = f(c + f(sc * f(int(qb.sum()))))
        corr[v] = f(64) * c
    for i, xr in enumerate(x):
        amax = f(np.nanmax(np.concatenate([[0], np.abs(xr)])))
        sx = amax / f(63) if amax > 0 else f(1)
        with np.errstate(invalid="ignore", divide="ignore"):
            xu = _clamp_cast(_round_half_away(xr / sx), -64, 63) + 64
        for v in range(vocab):
            acc = f(0)
            for b in range(nb):
                s = int(np.dot(xu[b * blk:(b + 1) * blk], q[v, b * blk:(b + 1) * blk]))
                acc = f(acc + f(f(s) * bs[v, b]))
            out[i, v] = f(f(acc - corr[v]) * sx)
    return q.astype(np.int8), bs, corr, out


def test_oracle_selects_a_row_within_quantization_error(oracle):
    # restates vocab_int8.rs:401-429 with seeded inputs
    rng = np.random.default_rng(7)
    w = rng.standard_normal((4096, 384), dtype=np.float32)
    x = rng.standard_normal((1, 384), dtype=np.float32)
    qw, bs, corr = oracle.int8_quantize(w, 32)
    ours = oracle.int8_gemv(x, qw, bs, corr, 32)[0]
    want = (x @ w.T)[0]
    picked, best = int(np.argmax(ours)), int(np.argmax(want))
    shortfall = (want[best] - want[picked]) / np.abs(want).max()
    assert shortfall < 0.02


@pytest.mark.parametrize("shape,blk", [((128, 20), 32), ((128, 96), 48), ((128, 96), 0),
                                       ((128, 96), 64), ((8, 64), -32)])
def test_oracle_declines_shapes_it_cannot_serve(oracle, shape, blk):
    # vocab_int8.rs:432-437 and the guard at :126-131
    w = np.ones(shape, np.float32)
    assert oracle.int8_quantize(w, blk) is None


@pytest.mark.parametrize("d,blk", [(96, 32), (96, 96), (192, 64), (192, 96)])
def test_oracle_matches_scalar_restatement(oracle, d, blk):
    rng = np.random.default_rng(d + blk)
    w = rng.standard_normal((9, d), dtype=np.float32)
    w[3] = 0.0  # zero row: every block scale 1
    w[5, :blk] = np.float32(0.5) * np.round(rng.uniform(-254, 254, blk)).astype(np.float32)
    w[5, 0] = 127.0  # block amax 127: scale 1, half-integer weights are ties
    x = rng.standard_normal((3, d), dtype=np.float32)
    x[1] = 0.0
    x[2] = np.float32(0.5) * np.round(rng.uniform(-126, 126, d)).astype(np.float32)
    x[2, 0] = 63.0  # sx = 1: half-integers are rounding ties
    q, bs, corr, out = _scalar_reference(w, x, blk)
    qw, obs, ocorr = oracle.int8_quantize(w, blk)
    assert np.array_equal(qw, q)
    assert np.array_equal(obs.view(np.int32), bs.view(np.int32))
    assert np.array_equal(ocorr.view(np.int32), corr.view(np.int32))
    got = oracle.int8_gemv(x, qw, obs, ocorr, blk, threads=2)
    assert np.array_equal(got.view(np.int32), out.view(np.int32))


def _nonfinite_case(d, blk, seed):
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((6, d), dtype=np.float32)
    w[1, 3] = np.nan            # ignored by the block maximum, quantised to 0
    w[2, blk + 1] = np.inf      # block scale inf: that row's output is not finite
    w[4, 5] = -np.inf
    x = rng.standard_normal((4, d), dtype=np.float32)
    x[0, 7] = np.nan            # quantised to 0 (+ 64)
    x[2, 1] = np.inf            # sx = inf
    x[3, :] = np.float32(1e-30)  # tiny: sx far below the normal range of the fast path
    x[3, 2] = np.float32(-2.5e-30)
    return w, x


def _same(a, b):
    """Bit-equal, NaN equal to NaN (payloads are the platform's)."""
    a, b = np.ascontiguousarray(a, np.float32), np.ascontiguousarray(b, np.float32)
    na, nb_ = np.isnan(a), np.isnan(b)
    return np.array_equal(na, nb_) and np.array_equal(a.view(np.int32)[~na], b.view(np.int32)[~nb_])


@pytest.mark.parametrize("d,blk", [(96, 32), (192, 64)])
def test_oracle_nonfinite_inputs(oracle, d, blk):
    w, x = _nonfinite_case(d, blk, d)
    q, bs, corr, out = _scalar_reference(w, x, blk)
    qw, obs, ocorr = oracle.int8_quantize(w, blk)
    assert np.array_equal(qw, q)
    assert _same(obs, bs) and _same(ocorr, corr)
    assert _same(oracle.int8_gemv(x, qw, obs, ocorr, blk, threads=1), out)


def test_abi_layout():
    from ffai_b200.int8_gemv import layout
    assert layout(51865, 1280, 32) == (3242 * 40 * 576, 51872)
    assert layout(384, 384, 96) == (24 * 4 * (96 * 16 + 64), 384)
    assert layout(1, 640, 640) == (640 * 16 + 64, 16)
    assert layout(100, 8192, 1024) == (7 * 8 * (1024 * 16 + 64), 112)
    for rows, cols, blk in [(8, 20, 32), (8, 384, 48), (8, 384, 0), (8, 384, -32), (8, 0, 32),
                            (0, 384, 32), (8, 2048, 2048), (8, 8224, 32)]:
        assert layout(rows, cols, blk) is None, (rows, cols, blk)


# --------------------------------------------------------------------------- GPU


def _weights(rows, cols, seed, ties=True):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.05))
    w[rows // 3] = 0.0  # zero row
    if rows > 7:
        w[7, :32] = 0.0  # one zero block
    if ties and rows > 11:
        w[11] = np.float32(0.5) * np.round(rng.uniform(-254, 254, cols)).astype(np.float32)
        w[11, ::32] = 127.0
    return w


def _acts(batch, cols, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((batch, cols), dtype=np.float32) * np.float32(3.0)
    if batch > 1:
        x[1] = 0.0  # zero activation row: sx = 1
    if batch > 2:
        x[2] = np.float32(0.5) * np.round(rng.uniform(-126, 126, cols)).astype(np.float32)
        x[2, 0] = -63.0
    return x


def _bits_equal(a, b):
    return np.array_equal(np.ascontiguousarray(a).view(np.int32), np.ascontiguousarray(b).view(np.int32))


@pytest.mark.gpu
@pytest.mark.parametrize("d,blk", [(384, 32), (1280, 64)])
def test_gemv_nonfinite_inputs(oracle, d, blk):
    from ffai_b200.int8_gemv import Int8Gemv
    w, x = _nonfinite_case(d, blk, d + 1)
    q = Int8Gemv.new(torch.from_numpy(w).to(DEV), blk)
    got = q.forward(torch.from_numpy(x).to(DEV)).cpu().numpy()
    qw, bs, corr = oracle.int8_quantize(w, blk)
    gq, gs, gc = (t.cpu().numpy() for t in q.unpacked())
    assert np.array_equal(gq, qw) and _same(gs, bs) and _same(gc, corr)
    assert _same(got, oracle.int8_gemv(x, qw, bs, corr, blk))


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols,blk,dtype", [
    (4096, 384, 32, torch.float32), (51865, 1280, 32, torch.float32),
    (5120, 1280, 64, torch.bfloat16), (1280, 5120, 32, torch.float16),
    (384, 384, 96, torch.float32), (1000, 1280, 640, torch.float32), (3, 640, 640, torch.float32),
    (100, 8192, 1024, torch.float32),
])
def test_quantize_matches_oracle(oracle, rows, cols, blk, dtype):
    from ffai_b200.int8_gemv import Int8Gemv
    w = torch.from_numpy(_weights(rows, cols, rows + cols)).to(dtype)
    q = Int8Gemv.new(w.to(DEV), blk)
    assert q is not None
    torch.cuda.synchronize()
    qw, bs, corr = oracle.int8_quantize(w.float().numpy(), blk)
    got_q, got_bs, got_corr = (t.cpu().numpy() for t in q.unpacked())
    assert np.array_equal(got_q, qw)
    assert _bits_equal(got_bs, bs)
    assert _bits_equal(got_corr, corr)
    # the padding rows of the last group are zero
    pq, ps, pc = q.unpacked(padded=True)
    assert pq.shape[0] - rows < 16
    assert not pq[rows:].any() and not ps[rows:].any() and not pc[rows:].any()


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols,blk", [
    (4096, 384, 32), (51865, 1280, 32), (51865, 384, 32), (5120, 1280, 64), (1280, 5120, 32),
    (384, 384, 96), (1280, 1280, 160), (1000, 1280, 640), (4097, 8192, 512), (3, 640, 640),
    (33, 64, 32), (600000, 64, 32), (2000, 8192, 1024), (1280, 1280, 32),
])
@pytest.mark.parametrize("batch", [1, 2, 3, 5, 8])
def test_gemv_matches_oracle(oracle, rows, cols, blk, batch):
    from ffai_b200.int8_gemv import Int8Gemv
    w = _weights(rows, cols, 3 * rows + cols)
    x = _acts(batch, cols, rows + batch)
    q = Int8Gemv.new(torch.from_numpy(w).to(DEV), blk)
    xd = torch.from_numpy(x).to(DEV)
    out = q.forward(xd)  # straight after the quantising kernel
    out2 = q.forward(xd)  # weights stable: streamed ahead of the preceding kernel's end
    torch.cuda.synchronize()
    assert torch.equal(out, out2)
    qw, bs, corr = oracle.int8_quantize(w, blk)
    want = oracle.int8_gemv(x, qw, bs, corr, blk)
    got = out.cpu().numpy()
    assert got.shape == (batch, rows)
    assert _bits_equal(got, want), f"max |diff| {np.abs(got - want).max()}"


@pytest.mark.gpu
def test_gemv_selects_a_row_within_quantization_error():
    # vocab_int8.rs:401-429 through the device path
    from ffai_b200.int8_gemv import Int8Gemv
    g = torch.Generator().manual_seed(11)
    w = torch.randn(4096, 384, generator=g)
    x = torch.randn(1, 384, generator=g)
    ours = Int8Gemv.new(w.to(DEV)).forward(x.to(DEV)).cpu()[0]
    want = (x @ w.T)[0]
    picked, best = int(ours.argmax()), int(want.argmax())
    assert (want[best] - want[picked]) / want.abs().max() < 0.02


@pytest.mark.gpu
def test_gemv_declines_and_rejects():
    from ffai_b200 import attention
    from ffai_b200.int8_gemv import Int8Gemv
    assert Int8Gemv.new(torch.randn(128, 20, device=DEV)) is None
    assert Int8Gemv.new(torch.randn(128, 96, device=DEV), blk=48) is None
    assert Int8Gemv.new(torch.randn(128, 96)) is None  # host tensor: not served here
    assert Int8Gemv.new(torch.randn(128, 2048, device=DEV), blk=2048) is None  # blk above 1024
    assert Int8Gemv.new(torch.randn(64, 8224, device=DEV)) is None  # wider than 8192
    q = Int8Gemv.new(torch.randn(64, 384, device=DEV))
    with pytest.raises(attention.AttnError) as e:
        q.forward(torch.randn(9, 384, device=DEV))
    assert e.value.status == _abi.ERR_INVALID
    with pytest.raises(TypeError):
        q.forward(torch.randn(1, 384, device=DEV, dtype=torch.bfloat16))

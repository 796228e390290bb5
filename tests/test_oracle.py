"""CPU tests of the oracle: the reference's own known-answer tests replayed
against the C++ restatement (flash_attn.rs:1000-1040), its exp polynomial,
its decode heads, and an f64 bound on its error.  No GPU needed."""

import numpy as np
import pytest

HD = 64


def _randn(rng, *shape, scale=1.0):
    return (rng.standard_normal(shape) * scale).astype(np.float32)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_matches_three_op_path(oracle, seed):
    """flash_attn.rs:1005-1021: H=4, seq=512, max |delta| < 1e-4 vs three-op."""
    rng = np.random.default_rng(seed)
    h, seq = 4, 512
    q = _randn(rng, 1, h, seq, HD)
    k = _randn(rng, 1, h, HD, seq)
    v = _randn(rng, 1, h, seq, HD)
    ours = oracle.attend(q, k, v, False)
    assert ours is not None, "the f32 encoder shape must be served"
    want = oracle.three_op(q, k, v)
    d = np.abs(ours - want).max()
    assert d < 1e-4, f"max |delta| {d:e} exceeds tolerance"


def test_declines_unsupported_shapes(oracle):
    """flash_attn.rs:1024-1039: one key at q_len 1, and masked attention."""
    rng = np.random.default_rng(0)
    q = _randn(rng, 1, 4, 1, HD)
    k = _randn(rng, 1, 4, HD, 1)
    v = _randn(rng, 1, 4, 1, HD)
    assert oracle.attend(q, k, v, False) is None
    q = _randn(rng, 1, 4, 512, HD)
    k = _randn(rng, 1, 4, HD, 512)
    v = _randn(rng, 1, 4, 512, HD)
    assert oracle.attend(q, k, v, True) is None


def test_decline_rules(oracle):
    rng = np.random.default_rng(1)
    # encoder shape below MIN_SEQ (flash_attn.rs:55) declines
    q = _randn(rng, 1, 2, 255, HD)
    k = _randn(rng, 1, 2, HD, 255)
    v = _randn(rng, 1, 2, 255, HD)
    assert oracle.attend(q, k, v, False) is None
    assert oracle.attend_merged(q, k, v) is None
    # q_len neither 1 nor keys declines
    q = _randn(rng, 1, 2, 300, HD)
    k = _randn(rng, 1, 2, HD, 400)
    v = _randn(rng, 1, 2, 400, HD)
    assert oracle.attend(q, k, v, False) is None
    # decode at the default floor (8 keys) is served, below it declines
    assert oracle.lib().ora_min_decode_keys() == 8
    q = _randn(rng, 1, 2, 1, HD)
    for keys, served in [(7, False), (8, True), (9, True)]:
        k = _randn(rng, 1, 2, HD, keys)
        v = _randn(rng, 1, 2, keys, HD)
        assert (oracle.attend(q, k, v, False) is not None) == served


def test_serves_predicate(oracle):
    """serves() requires keys >= max(MIN_SEQ, decode floor) (flash_attn.rs:112-128)."""
    assert oracle.serves((1, 6, 64, 1500), (1, 6, 1500, 64))
    assert not oracle.serves((1, 6, 64, 255), (1, 6, 255, 64))
    assert not oracle.serves((1, 6, 64, 1500), (1, 5, 1500, 64))
    assert not oracle.serves((2, 6, 64, 1500), (2, 6, 1500, 64))


def test_exp256_accuracy(oracle):
    """exp256 (flash_attn.rs:553-572).  Its coefficients are the Taylor
    coefficients of 2^f, so the truncated sixth-order term bounds the error at
    ln2^6/720 * 0.5^6 ~ 2.4e-6 relative (the reference's doc comment says
    ~1e-7); near the clamp the rounding of x*log2e adds a few e-6 more."""
    x = np.linspace(-87.0, 0.0, 8 * 4096, dtype=np.float32)
    y = oracle.exp256(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    rel = np.abs(y / ref - 1.0)
    assert rel.max() < 1e-5
    near = x > -10
    assert rel[near].max() < 4e-6
    clamp = oracle.exp256(np.full(8, -200.0, np.float32))
    assert np.allclose(clamp, np.exp(np.float64(-87.0)), rtol=1e-5)


@pytest.mark.parametrize("seq", [1, 7, 63, 64, 65, 255, 256, 257, 500])
def test_flash_head_any_length_vs_f64(oracle, seq):
    """flash_head is exact for any N (the 256 floor is a dispatch heuristic)."""
    rng = np.random.default_rng(seq)
    q = _randn(rng, seq, HD, scale=0.5 / 8)
    k = _randn(rng, seq, HD, scale=0.5)
    v = _randn(rng, seq, HD)
    out = oracle.flash_head(q, k.T.copy(), v)
    ref, _ = oracle.naive_attention_f64(q, k, v)
    assert np.abs(out - ref).max() < 2e-6


def test_merged_matches_heads_split(oracle):
    rng = np.random.default_rng(3)
    h, seq = 3, 300
    q = _randn(rng, 1, h, seq, HD, scale=0.1)
    k = _randn(rng, 1, h, HD, seq)
    v = _randn(rng, 1, h, seq, HD)
    a = oracle.attend(q, k, v, False)
    m = oracle.attend_merged(q, k, v)
    assert m.shape == (1, seq, h * HD)
    assert np.array_equal(m[0].reshape(seq, h, HD).transpose(1, 0, 2), a[0])


@pytest.mark.parametrize("keys", [1, 7, 8, 32, 128, 448, 1500])
def test_xattn_rows_vs_f64(oracle, keys):
    rng = np.random.default_rng(keys)
    rows = 6
    q = _randn(rng, rows, HD, scale=0.25)
    kt = _randn(rng, rows, HD, keys)
    v = _randn(rng, rows, keys, HD)
    out = oracle.xattn_rows(q, kt, v)
    ref, _ = oracle.naive_attention_f64(q[:, None, :], np.swapaxes(kt, 1, 2), v)
    assert np.abs(out - ref[:, 0]).max() < 2e-6


def test_xattn_f16_cache(oracle):
    rng = np.random.default_rng(11)
    rows, keys = 12, 1500
    q = _randn(rng, rows, HD, scale=0.25)
    kt = _randn(rng, rows, HD, keys).astype(np.float16)
    v = _randn(rng, rows, keys, HD).astype(np.float16)
    out = oracle.xattn_rows_f16(q, kt.view(np.uint16), v.view(np.uint16))
    ref, _ = oracle.naive_attention_f64(q[:, None, :], np.swapaxes(kt, 1, 2).astype(np.float64),
                                        v.astype(np.float64))
    assert np.abs(out - ref[:, 0]).max() < 2e-6
    # the f16 branch of attend serves only the decode shape
    out2 = oracle.attend_f16kv(q[None, :, None, :], kt[None].view(np.uint16), v[None].view(np.uint16))
    assert np.array_equal(out2[0, :, 0], out)


def test_bf16_round():
    from oracle import oracle as O
    x = np.array([1.0, 1.00390625, 1.005859375, -3.14159, 0.0, 65504.0], np.float32)
    r = O.bf16_round(x)
    import torch
    t = torch.from_numpy(x).to(torch.bfloat16).to(torch.float32).numpy()
    assert np.array_equal(r, t)

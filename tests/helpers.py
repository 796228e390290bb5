"""Shared comparison helpers for the parity tests (oracle on the host, the
library on the device, the same seeded inputs for both)."""

import numpy as np
import torch

# Tolerances of the parity bar (bf16 tensor-core path vs the oracle run in
# f32 on the same bf16-rounded inputs; checked f32 mode; softmax row sums).
BF16_MAX_ABS = 1e-2
BF16_MEAN_ABS = 1e-3
F32_REL = 1e-5
# Row sums of the softmax weights a kernel applies, measured directly with
# V = ones (then every output element is sum_j P_ij / l_i).
ROWSUM_TOL = 1e-6
# Consistency of the exported log-sum-exp with scores recomputed in f64: the
# kernels compute scores in f32 and store an f32 LSE (|lse| ~ 4-16, one ulp
# ~ 1e-6), so this check carries a ~1e-6 floor of its own.
LSE_TOL = 5e-6
# The tensor-core path normalises by the sum of the bf16/f16-rounded P it
# multiplies (so its applied weights sum to 1 within ROWSUM_TOL); its LSE is
# the log of that sum, within the rounding of P (~1e-4) of the exact value.
LSE_TC_TOL = 1e-3


def f32np(t: torch.Tensor) -> np.ndarray:
    return t.detach().to("cpu", torch.float32).contiguous().numpy()


def assert_bf16_close(got, ref, what=""):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    err = np.abs(got - ref)
    assert err.max() <= BF16_MAX_ABS, f"{what}: max |err| {err.max():.3e}"
    assert err.mean() <= BF16_MEAN_ABS, f"{what}: mean |err| {err.mean():.3e}"
    return err.max(), err.mean()


def assert_f32_close(got, ref, what=""):
    """Norm-wise relative error: max|got-ref| <= 1e-5 * max|ref|."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    rel = np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)
    assert rel <= F32_REL, f"{what}: relative error {rel:.3e}"
    return rel


def oracle_encoder(oracle, q, k, v, scale):
    """Oracle over (B,H,N,64) torch inputs (already rounded to their dtype):
    widen to f32, fold the scale into q as the reference's callers do, and run
    the restated flash_head per (sequence, head) on host threads.  The
    reference kernel only has the q_len == keys shape; other shapes are
    checked against the f64 textbook formula instead."""
    B, H, N, _ = q.shape
    if k.shape[2] != N:
        out, _ = oracle.naive_attention_f64(f32np(q), f32np(k), f32np(v), scale=scale)
        return out
    qn = f32np(q).reshape(B * H, N, 64)
    kn = f32np(k).reshape(B * H, k.shape[2], 64)
    vn = f32np(v).reshape(B * H, v.shape[2], 64)
    out = oracle.flash_rowmajor_k(qn, kn, vn, scale=scale)
    return out.reshape(B, H, N, 64)


def rowsum_error(q, k, scale, lse, rows=None):
    """max |sum_j exp(scale q_i.k_j - lse_i) - 1| in f64 (per (b,h) row set).

    q (U,N,64), k (U,M,64) f64-able arrays, lse (U,N)."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    lse = np.asarray(lse, np.float64)
    s = np.einsum("und,umd->unm", q, k) * scale
    tot = np.exp(s - lse[..., None]).sum(-1)
    return np.abs(tot - 1.0).max()

"""TEST INFRASTRUCTURE ONLY: numpy/ctypes front end of the CPU oracle.

The oracle is `flash_attn_ref.cpp`, a C++ restatement of the reference's AVX2
kernels in `crates/ffai-mercury/src/asr/flash_attn.rs` (see that file's
header).  Only `tests/`, `__graft_entry__.smoke()` and the CPU-baseline legs of
`bench.py` may import this module; the product package never does.

Parity pin: the reference's own tests for this path are the known answers
(`matches_three_op_path`, flash_attn.rs:1005-1021; `declines_unsupported_shapes`,
:1024-1039).  No golden vectors exist in the reference and the Rust reference
cannot be executed here, so parity is pinned to those tests.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HD = 64
MIN_SEQ = 256
OK, DECLINED = 0, 1

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "liboracle_flash.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (a few seconds with g++)."""
    if force or not os.path.exists(LIB_PATH):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        i = ctypes.c_int
        sig = {
            "ora_have_avx2": ([], i),
            "ora_have_f16c": ([], i),
            "ora_min_decode_keys": ([], i),
            "ora_exp256": ([_f32p, _f32p, i], None),
            "ora_flash_head_strided": ([_f32p, _f32p, _f32p, _f32p, i, i], None),
            "ora_flash_units": ([_f32p, _f32p, _f32p, _f32p, i, i, i], None),
            "ora_xattn_head": ([_f32p, _f32p, _f32p, _f32p, i], None),
            "ora_xattn_head_f16": ([_f32p, _u16p, _u16p, _f32p, i], None),
            "ora_xattn_rows": ([_f32p, _f32p, _f32p, _f32p, i, i, i], None),
            "ora_xattn_rows_f16": ([_f32p, _u16p, _u16p, _f32p, i, i, i], None),
            "ora_attend": ([_f32p, _f32p, _f32p, _f32p, i, i, i, i, i, i], i),
            "ora_attend_f16kv": ([_f32p, _u16p, _u16p, _f32p, i, i, i, i, i, i], i),
            "ora_attend_merged": ([_f32p, _f32p, _f32p, _f32p, i, i, i, i, i], i),
            "ora_serves": ([i] * 8, i),
            "ora_three_op": ([_f32p, _f32p, _f32p, _f32p, i, i, i], None),
            "ora_int8_quantize": ([_f32p, i, i, i, ctypes.c_void_p, _f32p, _f32p], i),
            "ora_int8_gemv": ([_f32p, i, ctypes.c_void_p, _f32p, _f32p, i, i, i, _f32p, i], None),
            "ora_f16_round": ([_f32p, ctypes.c_longlong, ctypes.c_void_p], None),
            "ora_fast_gelu": ([_f32p, _f32p, ctypes.c_longlong], None),
            "ora_f16_serves": ([i], i),
            "ora_f16_gemv": ([_f32p, i, ctypes.c_void_p, _f32p, i, i, _f32p, i], None),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def _f32(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a: np.ndarray, t=_f32p):
    return a.ctypes.data_as(t)


def default_threads() -> int:
    return max(1, os.cpu_count() or 1)


# --------------------------------------------------------------------------
# numeric helpers shared by tests and the bench
# --------------------------------------------------------------------------

def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round f32 -> bf16 (nearest-even) and widen back to f32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    out = (r & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    nan = np.isnan(x)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) of f32 values (nearest-even)."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def f16_round(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def naive_attention_f64(q, k, v, scale=1.0, causal=False, q_offset=0):
    """Textbook softmax(scale * q k^T) v in float64.

    q (..., Nq, D), k (..., Nk, D) row-major keys, v (..., Nk, D).  Used to
    bound the oracle's own error; it is not the parity reference.
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    s = np.einsum("...id,...jd->...ij", q, k) * scale
    if causal:
        nq, nk = s.shape[-2], s.shape[-1]
        allowed = np.arange(nk)[None, :] <= (q_offset + np.arange(nq))[:, None]
        s = np.where(allowed, s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(axis=-1, keepdims=True)
    lse = (m + np.log(l))[..., 0]
    return (p / l) @ v, lse


# --------------------------------------------------------------------------
# restated reference entry points
# --------------------------------------------------------------------------

def exp256(x: np.ndarray) -> np.ndarray:
    x = _f32(x)
    assert x.size % 8 == 0
    y = np.empty_like(x)
    lib().ora_exp256(_p(x), _p(y), x.size)
    return y


def flash_head(q, kt, v, out_stride=HD) -> np.ndarray:
    """One head: q (seq,64) pre-scaled, kt (64,seq), v (seq,64) -> (seq,64)."""
    q, kt, v = _f32(q), _f32(kt), _f32(v)
    seq = q.shape[0]
    if q.shape != (seq, HD) or kt.shape != (HD, seq) or v.shape != (seq, HD) or out_stride < HD:
        raise ValueError(f"flash_head shapes q {q.shape} kt {kt.shape} v {v.shape}")
    out = np.zeros((seq, out_stride), np.float32)
    lib().ora_flash_head_strided(_p(q), _p(kt), _p(v), _p(out), seq, out_stride)
    return out[:, :HD] if out_stride != HD else out


def flash_units(q, kt, v, threads=None) -> np.ndarray:
    """Many heads (units, seq, 64) with kt (units, 64, seq), on host threads."""
    q, kt, v = _f32(q), _f32(kt), _f32(v)
    if q.ndim != 3 or q.shape[2] != 64:
        raise ValueError(f"q must be (units, seq, 64), got {q.shape}")
    units, seq = q.shape[0], q.shape[1]
    if kt.shape != (units, 64, seq) or v.shape != (units, seq, 64):
        raise ValueError(f"kt {kt.shape} / v {v.shape} do not match q {q.shape}")
    out = np.empty_like(q)
    lib().ora_flash_units(_p(q), _p(kt), _p(v), _p(out), units, seq,
                          threads or default_threads())
    return out


def flash_rowmajor_k(q, k, v, scale=1.0, threads=None) -> np.ndarray:
    """Encoder attention for (units, seq, 64) q/k/v with row-major k.

    Folds `scale` into q first, as the reference's callers do before the
    kernel (text_decoder.rs:827-844), and transposes k into the kernel's
    head-dim-major K^T layout.
    """
    q = _f32(np.asarray(q, np.float32) * np.float32(scale))
    kt = _f32(np.swapaxes(np.asarray(k, np.float32), -1, -2))
    return flash_units(q, kt, v, threads)


def xattn_rows(q, kt, v, threads=1) -> np.ndarray:
    """Decode rows: q (rows,64), kt (rows,64,keys), v (rows,keys,64), f32."""
    q, kt, v = _f32(q), _f32(kt), _f32(v)
    rows, keys = q.shape[0], kt.shape[-1]
    if q.shape != (rows, HD) or kt.shape != (rows, HD, keys) or v.shape != (rows, keys, HD):
        raise ValueError(f"xattn_rows shapes q {q.shape} kt {kt.shape} v {v.shape}")
    out = np.empty((rows, HD), np.float32)
    lib().ora_xattn_rows(_p(q), _p(kt), _p(v), _p(out), rows, keys, threads)
    return out


def xattn_rows_f16(q, kt_bits, v_bits, threads=1) -> np.ndarray:
    """Decode rows over an f16 cache given as uint16 bit patterns."""
    q = _f32(q)
    kt_bits = np.ascontiguousarray(kt_bits, np.uint16)
    v_bits = np.ascontiguousarray(v_bits, np.uint16)
    rows, keys = q.shape[0], kt_bits.shape[-1]
    if q.shape != (rows, HD) or kt_bits.shape != (rows, HD, keys) or v_bits.shape != (rows, keys, HD):
        raise ValueError(f"xattn_rows_f16 shapes q {q.shape} kt {kt_bits.shape} v {v_bits.shape}")
    out = np.empty((rows, HD), np.float32)
    lib().ora_xattn_rows_f16(_p(q), _p(kt_bits, _u16p), _p(v_bits, _u16p), _p(out), rows, keys,
                             threads)
    return out


def attend(q, kt, v, masked=False, threads=1):
    """flash_attn::attend (f32): returns the output, or None when declined.

    q (1,H,qlen,64), kt (1,H,64,keys), v (1,H,keys,64) -> (1,H,qlen,64).
    """
    q, kt, v = _f32(q), _f32(kt), _f32(v)
    _, h, qlen, hd = q.shape
    keys = kt.shape[-1]
    if kt.shape != (1, h, hd, keys) or v.shape != (1, h, keys, hd):
        return None
    out = np.zeros((1, h, qlen, HD), np.float32)
    st = lib().ora_attend(_p(q), _p(kt), _p(v), _p(out), h, qlen, keys, hd, int(masked), threads)
    return None if st == DECLINED else out


def attend_f16kv(q, kt_bits, v_bits, masked=False, threads=1):
    q = _f32(q)
    kt_bits = np.ascontiguousarray(kt_bits, np.uint16)
    v_bits = np.ascontiguousarray(v_bits, np.uint16)
    _, h, qlen, hd = q.shape
    keys = kt_bits.shape[-1]
    out = np.zeros((1, h, qlen, HD), np.float32)
    st = lib().ora_attend_f16kv(_p(q), _p(kt_bits, _u16p), _p(v_bits, _u16p), _p(out), h, qlen,
                                keys, hd, int(masked), threads)
    return None if st == DECLINED else out


def attend_merged(q, kt, v, threads=1):
    """flash_attn::attend_merged: (1,H,N,64) operands -> (1,N,H*64) or None."""
    q, kt, v = _f32(q), _f32(kt), _f32(v)
    _, h, qlen, hd = q.shape
    keys = kt.shape[-1]
    if kt.shape != (1, h, hd, keys) or v.shape != (1, h, keys, hd):
        return None
    out = np.zeros((1, qlen, h * HD), np.float32)
    st = lib().ora_attend_merged(_p(q), _p(kt), _p(v), _p(out), h, qlen, keys, hd, threads)
    return None if st == DECLINED else out


def serves(kt_shape, v_shape) -> bool:
    return bool(lib().ora_serves(*[int(x) for x in kt_shape], *[int(x) for x in v_shape]))


def three_op(q, kt, v) -> np.ndarray:
    """softmax_last_dim(q @ kt) @ v in f32, the reference test's comparator."""
    q, kt, v = _f32(q), _f32(kt), _f32(v)
    _, h, qlen, _ = q.shape
    keys = kt.shape[-1]
    out = np.empty((1, h, qlen, HD), np.float32)
    lib().ora_three_op(_p(q), _p(kt), _p(v), _p(out), h, qlen, keys)
    return out


# --------------------------------------------------------------------------
# int8 GEMV (vocab_int8.rs), restated in vocab_int8_ref.cpp
# --------------------------------------------------------------------------

def int8_quantize(w, blk=32):
    """Int8Vocab::new: w (vocab, d) -> (qw int8, bscale f32, corr f32), or
    None when the shape is not served (blk or d not multiples as required)."""
    w = _f32(w)
    vocab, d = w.shape
    qw = np.empty((vocab, d), np.int8)
    nb = d // blk if blk > 0 and d % blk == 0 else 1
    bscale = np.empty((vocab, nb), np.float32)
    corr = np.empty(vocab, np.float32)
    st = lib().ora_int8_quantize(_p(w), vocab, d, blk, qw.ctypes.data_as(ctypes.c_void_p),
                                 _p(bscale), _p(corr))
    if st != 0:
        return None
    return qw, bscale, corr


def int8_gemv(x, qw, bscale, corr, blk=32, threads=None):
    """Int8VocabOp::cpu_fwd per activation row: x (batch, d) -> (batch, vocab)."""
    x = _f32(np.atleast_2d(x))
    vocab, d = qw.shape
    qw = np.ascontiguousarray(qw, np.int8)
    out = np.empty((x.shape[0], vocab), np.float32)
    lib().ora_int8_gemv(_p(x), x.shape[0], qw.ctypes.data_as(ctypes.c_void_p), _p(_f32(bscale)),
                        _p(_f32(corr)), vocab, d, blk, _p(out), threads or default_threads())
    return out


# --------------------------------------------------------------------------
# f16 GEMV (f16_gemv.rs), restated in f16_gemv_ref.cpp
# --------------------------------------------------------------------------

def f16_weights(w):
    """F16Gemv::new's weights: f32 -> f16 bits (nearest-even), same shape, uint16;
    None when the shape is not served (cols not a multiple of 8)."""
    w = _f32(w)
    if w.ndim != 2 or lib().ora_f16_serves(w.shape[1]) != 0:
        return None
    out = np.empty(w.shape, np.uint16)
    lib().ora_f16_round(_p(w), w.size, out.ctypes.data_as(ctypes.c_void_p))
    return out


def f16_gemv(x, w16, bias=None, threads=None):
    """dot_f16 per activation row (+ bias after): x (batch, cols) -> (batch, rows)."""
    x = _f32(np.atleast_2d(x))
    w16 = np.ascontiguousarray(w16, np.uint16)
    rows, cols = w16.shape
    out = np.empty((x.shape[0], rows), np.float32)
    b = None if bias is None else _f32(bias)
    lib().ora_f16_gemv(_p(x), x.shape[0], w16.ctypes.data_as(ctypes.c_void_p),
                       None if b is None else _p(b), rows, cols, _p(out), threads or default_threads())
    return out


# --------------------------------------------------------------------------
# FastGelu (text_decoder.rs gelu_scalar), restated in fast_gelu_ref.cpp
# --------------------------------------------------------------------------

def fast_gelu(x):
    """gelu_scalar elementwise, f32 in, f32 out."""
    x = _f32(x)
    y = np.empty_like(x)
    lib().ora_fast_gelu(_p(x), _p(y), x.size)
    return y


"""ctypes binding of include/ffai_attn.h (the C ABI of libffai_attn.so).

This is the Python counterpart of the `extern "C"` block a Rust crate would
declare for the same library.  Loading fails loudly when the shared library
has not been built: there is no CPU fallback behind this module.
"""

from __future__ import annotations

import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libffai_attn.so")

# status codes
OK = 0
DECLINED = 1
ERR_INVALID = -1
ERR_CUDA = -2
ERR_TIMEOUT = -3
ERR_NOMEM = -4
ERR_NO_DEVICE = -5

# dtypes
DT_F32, DT_BF16, DT_F16 = 0, 1, 2
# layouts
LAYOUT_HEADS_SPLIT, LAYOUT_TOKEN_MAJOR, LAYOUT_KT = 0, 1, 2
# flags
FLAG_CHECKED_F32 = 0x1
FLAG_KV_STABLE = 0x2
FLAG_KV_APPEND_ONLY = 0x4
FLAG_INPUTS_STABLE = 0x8
# ops
OP_PREFILL, OP_DECODE, OP_VARLEN = 0, 1, 2


class Desc(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("q_len", ctypes.c_int32),
        ("kv_len", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("kv_capacity", ctypes.c_int32),
        ("q_dtype", ctypes.c_int32),
        ("kv_dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
        ("q_layout", ctypes.c_int32),
        ("k_layout", ctypes.c_int32),
        ("v_layout", ctypes.c_int32),
        ("out_layout", ctypes.c_int32),
        ("causal", ctypes.c_int32),
        ("q_offset", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("flags", ctypes.c_uint32),
        ("token_stride", ctypes.c_int32),
    ]


class Tensor4(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dims", ctypes.c_int64 * 4),
        ("dtype", ctypes.c_int32),
        ("device", ctypes.c_int32),
    ]


# every symbol include/ffai_attn.h declares, with (argtypes, restype)
_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_DescP = ctypes.POINTER(Desc)
_T4P = ctypes.POINTER(Tensor4)
_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)

SIGNATURES = {
    "ffai_attn_version": ([], ctypes.c_char_p),
    "ffai_attn_desc_init": ([_DescP], None),
    "ffai_attn_check": ([_DescP, ctypes.c_int], ctypes.c_int),
    "ffai_attn_create": ([ctypes.c_int, ctypes.POINTER(ctypes.c_int)], _vp),
    "ffai_attn_destroy": ([_vp], None),
    "ffai_attn_prefill": ([_vp, _DescP, _vp, _vp, _vp, _vp, _vp, _vp], ctypes.c_int),
    "ffai_attn_decode": ([_vp, _DescP, _vp, _vp, _vp, _vp, _vp, _i32, _vp], ctypes.c_int),
    "ffai_attn_decode_prefetch": ([_vp, _DescP, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
                                  ctypes.c_int),
    "ffai_attn_decode_static": ([_DescP, _vp, _vp, _vp, _vp, _vp, _i32, _vp], ctypes.c_int),
    "ffai_attn_multi_prefill_host": ([ctypes.POINTER(_vp), _i32, _DescP, _vp, _vp, _vp, _vp, _vp,
                                      _i32, _i32p], ctypes.c_int),
    "ffai_attn_chunk_queue_selftest": ([_i32, _i32, ctypes.c_uint32, _i32p, _i32p], ctypes.c_int),
    "ffai_attn_decode_paged": ([_vp, _DescP, _vp, _vp, _vp, _i32, _vp, _vp, _i32, _vp, _vp, _vp],
                               ctypes.c_int),
    "ffai_kv_append": ([_vp, _DescP, _vp, _vp, _i32, _vp, _vp, _i32, _vp, _vp, _vp], ctypes.c_int),
    "ffai_kv_copy_pages": ([_vp, _DescP, _vp, _vp, _i32, _vp, _vp, _i32, _vp], ctypes.c_int),
    "ffai_int8_gemv_layout": ([_i32, _i32, _i32, _vp, _vp], ctypes.c_int),
    "ffai_f16_gemv_layout": ([_i32, _i32, _vp], ctypes.c_int),
    "ffai_gemm_bf16": ([_vp, _vp, ctypes.c_int64, _vp, ctypes.c_int64, _vp, _vp, ctypes.c_int64,
                        _vp, ctypes.c_int64, _i32, _i32, _i32, _i32, _i32, _vp], ctypes.c_int),
    "ffai_f16_gemv_pack": ([_vp, _vp, _i32, _i32, _i32, _vp, _vp], ctypes.c_int),
    "ffai_f16_gemv": ([_vp, _vp, _i32, _vp, _vp, _i32, _i32, _vp, ctypes.c_uint32, _vp],
                      ctypes.c_int),
    "ffai_int8_gemv_quantize": ([_vp, _vp, _i32, _i32, _i32, _i32, _vp, _vp, _vp], ctypes.c_int),
    "ffai_int8_gemv": ([_vp, _vp, _i32, _vp, _vp, _i32, _i32, _i32, _vp, ctypes.c_uint32, _vp],
                       ctypes.c_int),
    "ffai_attn_profile": ([_vp, _i32, ctypes.POINTER(ctypes.c_double),
                           ctypes.POINTER(ctypes.c_int64)], ctypes.c_int),
    "ffai_attn_varlen": ([_vp, _DescP, _i32p, _i32p, _i32, _vp, _vp, _vp, _vp, _vp, _vp],
                         ctypes.c_int),
    "ffai_attn_prefill_host": ([_vp, _DescP, _vp, _vp, _vp, _vp, _vp], ctypes.c_int),
    "ffai_attn_sync": ([_vp, _vp], ctypes.c_int),
    "ffai_attn_last_error": ([_vp, ctypes.c_char_p, ctypes.c_size_t], ctypes.c_int),
    "ffai_flash_serves": ([_T4P, _T4P], ctypes.c_int),
    "ffai_flash_attend": ([_vp, _T4P, _T4P, _T4P, _i32, _T4P, _vp], ctypes.c_int),
    "ffai_flash_attend_merged": ([_vp, _T4P, _T4P, _T4P, _T4P, _vp], ctypes.c_int),
    "ffai_flash_check": ([_T4P, _T4P, _T4P, _i32, _i32], ctypes.c_int),
}

_lib = None


def load() -> ctypes.CDLL:
    """Load libffai_attn.so and declare every entry point; raise if absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is not built; run `python -m ffai_b200.build` "
                "(this package has no CPU fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
    return _lib


def last_error(ctx=None) -> str:
    buf = ctypes.create_string_buffer(512)
    load().ffai_attn_last_error(ctx, buf, len(buf))
    return buf.value.decode(errors="replace")


def new_desc(**kw) -> Desc:
    d = Desc()
    load().ffai_attn_desc_init(ctypes.byref(d))
    for k, v in kw.items():
        setattr(d, k, v)
    return d

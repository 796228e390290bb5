"""CPU tests of the C-ABI boundary: libffai_attn.so loads, exports every
function include/ffai_attn.h declares, agrees with the header's struct
layout, and applies the shape/dtype gate (the reference's decline contract)
without a GPU."""

import ctypes
import os
import re
import subprocess

import pytest

from ffai_b200 import _abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ffai_attn.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"\b(ffai_\w+)\s*\(", text)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    from ffai_b200 import build
    build.build()
    return _abi.load()


def test_exports_every_declared_symbol(lib):
    names = header_functions()
    assert len(names) >= 14
    for n in names:
        assert hasattr(lib, n), f"{n} declared in ffai_attn.h but not exported"
    # and the Python binding declares exactly the header's functions
    assert sorted(_abi.SIGNATURES) == names


def test_version(lib):
    assert lib.ffai_attn_version().decode().startswith("ffai-attn-b200")


def test_struct_layout_matches_header(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "ffai_attn.h"\n'
        "int main(void){printf(\"%zu %zu %zu %zu %zu %zu %zu\\n\","
        "sizeof(ffai_attn_desc), offsetof(ffai_attn_desc, scale), offsetof(ffai_attn_desc, flags),"
        "sizeof(ffai_tensor4), offsetof(ffai_tensor4, dims), offsetof(ffai_tensor4, dtype),"
        "offsetof(ffai_tensor4, device));return 0;}\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-I", os.path.dirname(HEADER), str(src), "-o", str(exe)],
                   check=True)
    got = [int(x) for x in subprocess.check_output([str(exe)]).split()]
    want = [ctypes.sizeof(_abi.Desc), _abi.Desc.scale.offset, _abi.Desc.flags.offset,
            ctypes.sizeof(_abi.Tensor4), _abi.Tensor4.dims.offset, _abi.Tensor4.dtype.offset,
            _abi.Tensor4.device.offset]
    assert got == want


def _check(lib, op=_abi.OP_PREFILL, **kw):
    d = _abi.new_desc(**kw)
    return lib.ffai_attn_check(ctypes.byref(d), op)


def test_check_gate(lib):
    enc = dict(batch=8, heads=8, q_len=1500, kv_len=1500, q_dtype=_abi.DT_BF16,
               kv_dtype=_abi.DT_BF16, scale=0.125)
    assert _check(lib, **enc) == _abi.OK
    assert _check(lib, **{**enc, "head_dim": 128}) == _abi.DECLINED
    assert _check(lib, **{**enc, "kv_dtype": _abi.DT_F16}) == _abi.DECLINED
    assert _check(lib, **{**enc, "q_len": 0}) == _abi.ERR_INVALID
    assert _check(lib, **{**enc, "scale": 0.0}) == _abi.ERR_INVALID
    assert _check(lib, **{**enc, "kv_capacity": 100}) == _abi.ERR_INVALID
    assert _check(lib, **{**enc, "q_layout": _abi.LAYOUT_KT}) == _abi.ERR_INVALID
    # causal prefill: tensor-core and checked f32 kernels; q_offset >= 0
    assert _check(lib, **{**enc, "causal": 1}) == _abi.OK
    assert _check(lib, **{**enc, "causal": 1, "q_offset": -1}) == _abi.ERR_INVALID
    f32 = dict(enc, q_dtype=_abi.DT_F32, kv_dtype=_abi.DT_F32)
    assert _check(lib, **{**f32, "causal": 1, "flags": _abi.FLAG_CHECKED_F32}) == _abi.OK
    assert _check(lib, **{**enc, "flags": _abi.FLAG_CHECKED_F32}) == _abi.DECLINED
    # decode
    dec = dict(batch=5, heads=12, q_len=1, kv_len=1500, q_dtype=_abi.DT_F32,
               kv_dtype=_abi.DT_BF16, k_layout=_abi.LAYOUT_KT)
    assert _check(lib, _abi.OP_DECODE, **dec) == _abi.OK
    assert _check(lib, _abi.OP_DECODE, **{**dec, "q_len": 2}) == _abi.DECLINED
    assert _check(lib, _abi.OP_DECODE, **{**dec, "q_dtype": _abi.DT_F16}) == _abi.DECLINED
    assert _check(lib, _abi.OP_DECODE, **{**dec, "v_layout": _abi.LAYOUT_TOKEN_MAJOR}) == _abi.DECLINED
    # the decode kernels read q and write out as dense rows: a fused-projection
    # view (token_stride set) is declined rather than misread
    assert _check(lib, _abi.OP_DECODE, **{**dec, "token_stride": 3 * 12 * 64}) == _abi.DECLINED
    assert "token_stride" in _abi.last_error(None)
    # varlen
    tm = _abi.LAYOUT_TOKEN_MAJOR
    var = dict(heads=16, q_dtype=_abi.DT_BF16, kv_dtype=_abi.DT_BF16, q_layout=tm, k_layout=tm,
               v_layout=tm, out_layout=tm)
    assert _check(lib, _abi.OP_VARLEN, **var) == _abi.OK
    assert _check(lib, _abi.OP_VARLEN, **{**var, "q_layout": 0}) == _abi.DECLINED
    assert _check(lib, _abi.OP_VARLEN, **{**var, "q_dtype": 0, "kv_dtype": 0}) == _abi.DECLINED
    assert _check(lib, 7, **enc) == _abi.ERR_INVALID
    assert "unknown op" in _abi.last_error(None)


def test_create_without_device_fails_cleanly(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    st = ctypes.c_int(123)
    ctx = lib.ffai_attn_create(0, ctypes.byref(st))
    assert not ctx
    assert st.value == _abi.ERR_NO_DEVICE
    assert lib.ffai_attn_prefill(None, None, None, None, None, None, None, None) == _abi.ERR_INVALID


def test_serves_on_host_tensors_declines(lib):
    kt = _abi.Tensor4(None, (ctypes.c_int64 * 4)(1, 6, 64, 1500), _abi.DT_F32, -1)
    v = _abi.Tensor4(None, (ctypes.c_int64 * 4)(1, 6, 1500, 64), _abi.DT_F32, -1)
    assert lib.ffai_flash_serves(ctypes.byref(kt), ctypes.byref(v)) == 0
    kt.device = v.device = 0
    assert lib.ffai_flash_serves(ctypes.byref(kt), ctypes.byref(v)) == 1
    kt.dims[3] = v.dims[2] = 255  # below MIN_SEQ (flash_attn.rs:112-128)
    assert lib.ffai_flash_serves(ctypes.byref(kt), ctypes.byref(v)) == 0


def test_flash_check_applies_the_reference_decline_rules(lib):
    """ffai_flash_check: attend / attend_merged's decision on the operands
    alone (flash_attn.rs:135-158, :218-264), without a context or a GPU."""
    def t4(dims, dt=_abi.DT_F32, dev=0):
        return _abi.Tensor4(None, (ctypes.c_int64 * 4)(*dims), dt, dev)

    def check(q, kt, v, masked=0, merged=0):
        return lib.ffai_flash_check(ctypes.byref(q), ctypes.byref(kt), ctypes.byref(v),
                                    masked, merged)

    enc = (t4((1, 6, 1500, 64)), t4((1, 6, 64, 1500)), t4((1, 6, 1500, 64)))
    assert check(*enc) == _abi.OK
    assert check(*enc, merged=1) == _abi.OK
    assert check(*enc, masked=1) == _abi.DECLINED
    # below MIN_SEQ at the encoder shape
    short = (t4((1, 6, 200, 64)), t4((1, 6, 64, 200)), t4((1, 6, 200, 64)))
    assert check(*short) == _abi.DECLINED
    # decode shape: 16-bit caches are served, not at the encoder shape or merged
    dec = (t4((1, 12, 1, 64)), t4((1, 12, 64, 1500), _abi.DT_F16), t4((1, 12, 1500, 64), _abi.DT_F16))
    assert check(*dec) == _abi.OK
    assert check(*dec, merged=1) == _abi.DECLINED
    half_enc = (enc[0], t4((1, 6, 64, 1500), _abi.DT_BF16), t4((1, 6, 1500, 64), _abi.DT_BF16))
    assert check(*half_enc) == _abi.DECLINED
    # q_len neither 1 nor keys; host memory; mixed devices
    mid = (t4((1, 6, 700, 64)), enc[1], enc[2])
    assert check(*mid) == _abi.DECLINED
    assert check(t4((1, 6, 1500, 64), dev=-1), *enc[1:]) == _abi.DECLINED
    assert check(enc[0], t4((1, 6, 64, 1500), dev=1), enc[2]) == _abi.DECLINED
    assert "device" in _abi.last_error(None)


def test_python_flag_constants_match_the_header():
    text = open(HEADER).read()
    defines = {n: int(v, 0) for n, v in
               re.findall(r"#define FFAI_ATTN_(FLAG_\w+) (0x[0-9a-fA-F]+)u", text)}
    assert set(defines) == {"FLAG_CHECKED_F32", "FLAG_KV_STABLE", "FLAG_KV_APPEND_ONLY",
                            "FLAG_INPUTS_STABLE"}
    for name, value in defines.items():
        assert getattr(_abi, name) == value, name

"""CPU checks that the Rust crate binding the library (crates/ffai-attn-sys)
stays in step with include/ffai_attn.h, since this image has no Rust
toolchain to compile it: every `extern "C"` function, `#[repr(C)]` struct and
constant of src/lib.rs is compared with the header (names, argument and
field order, C types), build.rs must compile every CUDA source the Python
build compiles (it lists the directory rather than naming files), and the
patch to the reference's flash_attn.rs applies to the reference's sources
when they are present."""

import os
import re
import shutil
import subprocess

import pytest

from ffai_b200 import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ffai_attn.h")
CRATE = os.path.join(ROOT, "crates", "ffai-attn-sys")
LIB_RS = os.path.join(CRATE, "src", "lib.rs")
REFERENCE = "/root/reference"

C_TYPES = {"int32_t": "i32", "int": "i32", "uint32_t": "u32", "int64_t": "i64", "float": "f32",
           "double": "f64", "size_t": "usize"}
RUST_TYPES = {"i32": "i32", "c_int": "i32", "u32": "u32", "i64": "i64", "f32": "f32",
              "f64": "f64", "usize": "usize"}


def _strip_c(text):
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.sub(r"//[^\n]*", "", text)


def _c_class(decl):
    decl = decl.strip()
    if "*" in decl:
        return "ptr"
    words = decl.replace("const ", "").split()
    return C_TYPES[words[0]] if words else "void"


def _rust_class(ty):
    ty = ty.strip()
    if ty.startswith("*"):
        return "ptr"
    return RUST_TYPES[ty]


def header_functions():
    text = _strip_c(open(HEADER).read())
    text = "\n".join(l for l in text.splitlines() if not l.lstrip().startswith("#"))
    out = {}
    for m in re.finditer(r"^([A-Za-z_][\w \t\*]*?)\b(ffai_\w+)\s*\(([^)]*)\)\s*;", text,
                         flags=re.M):
        ret, name, params = m.group(1), m.group(2), m.group(3).strip()
        args = [] if params in ("", "void") else [_c_class(p) for p in params.split(",")]
        out[name] = (args, "void" if ret.strip() == "void" else _c_class(ret))
    return out


def rust_functions():
    text = open(LIB_RS).read()
    block = re.search(r'unsafe extern "C" \{(.*?)\n\}', text, flags=re.S).group(1)
    out = {}
    for m in re.finditer(r"pub fn (\w+)\((.*?)\)\s*(?:->\s*([^;]+))?;", block, flags=re.S):
        name, params, ret = m.group(1), m.group(2).strip(), m.group(3)
        args = []
        if params:
            for p in re.split(r",\s*(?![^()]*\))", params):
                if p.strip():
                    args.append(_rust_class(p.split(":", 1)[1]))
        out[name] = (args, "void" if ret is None else _rust_class(ret))
    return out


def header_struct(name):
    text = _strip_c(open(HEADER).read())
    body = re.search(r"typedef struct %s \{(.*?)\}" % name, text, flags=re.S).group(1)
    fields = []
    for decl in body.split(";"):
        decl = decl.strip()
        if not decl:
            continue
        m = re.match(r"(.*?)\s*(\**)\s*(\w+)\s*(\[\d+\])?$", decl)
        ctype, star, fname, arr = m.groups()
        cls = "ptr" if star else C_TYPES[ctype.split()[-1]]
        fields.append((fname, cls + (arr or "")))
    return fields


def rust_struct(name):
    text = open(LIB_RS).read()
    body = re.search(r"pub struct %s \{(.*?)\n\}" % name, text, flags=re.S).group(1)
    fields = []
    for fname, ty in re.findall(r"pub (\w+):\s*([^,\n]+),", body):
        ty = ty.strip()
        arr = re.match(r"\[(\w+);\s*(\d+)\]", ty)
        fields.append((fname, RUST_TYPES[arr.group(1)] + f"[{arr.group(2)}]" if arr
                       else _rust_class(ty)))
    return fields


def test_every_header_function_is_bound_with_the_same_signature():
    h, r = header_functions(), rust_functions()
    assert len(h) >= 29
    assert sorted(h) == sorted(r), (sorted(set(h) ^ set(r)))
    for name in h:
        assert h[name] == r[name], f"{name}: header {h[name]} vs lib.rs {r[name]}"


@pytest.mark.parametrize("name", ["ffai_attn_desc", "ffai_tensor4"])
def test_repr_c_structs_match_the_header(name):
    assert header_struct(name) == rust_struct(name)


def test_constants_match_the_header():
    text = _strip_c(open(HEADER).read())
    defines = {}
    for n, v in re.findall(r"#define (FFAI_\w+) \(?(-?(?:0x)?[0-9a-fA-F]+)u?\)?", text):
        defines[n] = int(v, 0)
    rust = {n: int(v.replace("_", ""), 0)
            for n, v in re.findall(r"pub const (FFAI_\w+): \w+ = (-?(?:0x)?[0-9a-fA-F_]+);",
                                   open(LIB_RS).read())}
    assert len(defines) >= 20
    assert defines == rust


def test_build_rs_compiles_every_cuda_source():
    src = open(os.path.join(CRATE, "build.rs")).read()
    # no hand-kept list: the directory is listed, by extension
    assert not re.search(r'"\w+\.cu"', src)
    assert "read_dir" in src and '== "cu"' in src
    assert "compute_100a,code=sm_100a" in src
    on_disk = sorted(f for f in os.listdir(build.CSRC) if f.endswith(".cu"))
    assert build.SOURCES == on_disk


@pytest.mark.skipif(not os.path.isdir(REFERENCE), reason="reference sources not present")
def test_patch_applies_to_the_reference(tmp_path):
    for rel in ("crates/ffai-mercury/Cargo.toml", "crates/ffai-mercury/src/asr/flash_attn.rs"):
        dst = tmp_path / rel
        dst.parent.mkdir(parents=True, exist_ok=True)
        shutil.copy(os.path.join(REFERENCE, rel), dst)
    subprocess.run(["git", "init", "-q"], cwd=tmp_path, check=True)
    patch = os.path.join(CRATE, "patches", "flash_attn_cuda.patch")
    subprocess.run(["git", "apply", "--unidiff-zero", patch], cwd=tmp_path, check=True)
    fa = (tmp_path / "crates/ffai-mercury/src/asr/flash_attn.rs").read_text()
    for fn in ("serves(kt, v)", "attend_merged(q, kt, v)", "attend(q, kt, v, masked)"):
        assert f"ffai_attn_sys::candle_ops::{fn}" in fa
    # every function the patch calls exists in the crate's candle glue
    glue = open(os.path.join(CRATE, "src", "candle_ops.rs")).read()
    for fn in ("serves", "attend_merged", "attend"):
        assert re.search(r"pub fn %s\(" % fn, glue)

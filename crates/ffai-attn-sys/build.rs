//! Compiles every CUDA source of the library for sm_100a into a static
//! archive and links it (with the static CUDA runtime) into the crate.
//!
//! The sources are found by listing the directory, not from a list kept
//! here, so a file added to the library cannot be left out of this build:
//! every `*.cu` under the source directory is compiled.
//!
//! Environment:
//!   FFAI_ATTN_CSRC  directory of the `.cu` sources (default: the
//!                   repository's `ffai_b200/csrc`, two levels up)
//!   NVCC            the compiler (default: `$CUDA_HOME/bin/nvcc`, else `nvcc`)
//!   CUDA_HOME       toolkit root for `lib64/libcudart_static.a`
//!                   (default `/usr/local/cuda`)

use std::env;
use std::path::{Path, PathBuf};
use std::process::Command;

fn cuda_sources(dir: &Path) -> Vec<PathBuf> {
    let mut srcs: Vec<PathBuf> = std::fs::read_dir(dir)
        .unwrap_or_else(|e| panic!("ffai-attn-sys: cannot list {}: {e}", dir.display()))
        .filter_map(Result::ok)
        .map(|e| e.path())
        .filter(|p| p.extension().is_some_and(|x| x == "cu"))
        .collect();
    srcs.sort();
    assert!(!srcs.is_empty(), "ffai-attn-sys: no .cu sources in {}", dir.display());
    srcs
}

fn main() {
    let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap());
    let csrc = env::var_os("FFAI_ATTN_CSRC")
        .map(PathBuf::from)
        .unwrap_or_else(|| manifest.join("../../ffai_b200/csrc"));
    let include = csrc.join("../../include");
    let cuda_home = env::var("CUDA_HOME").unwrap_or_else(|_| "/usr/local/cuda".into());
    let nvcc = env::var("NVCC").unwrap_or_else(|_| {
        let p = Path::new(&cuda_home).join("bin/nvcc");
        if p.exists() { p.display().to_string() } else { "nvcc".into() }
    });
    let out = PathBuf::from(env::var("OUT_DIR").unwrap());

    println!("cargo:rerun-if-env-changed=FFAI_ATTN_CSRC");
    println!("cargo:rerun-if-env-changed=NVCC");
    println!("cargo:rerun-if-env-changed=CUDA_HOME");
    println!("cargo:rerun-if-changed={}", csrc.display());
    for e in std::fs::read_dir(&csrc).unwrap().filter_map(Result::ok) {
        println!("cargo:rerun-if-changed={}", e.path().display());
    }
    println!("cargo:rerun-if-changed={}", include.join("ffai_attn.h").display());

    // One object per source, then one archive: no relocatable device code
    // crosses files, so the archive links like any host library.
    let mut objs = Vec::new();
    for src in cuda_sources(&csrc) {
        let obj = out.join(src.file_stem().unwrap()).with_extension("o");
        let st = Command::new(&nvcc)
            .args(["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo",
                   "-std=c++17", "-Xcompiler", "-fPIC", "-c"])
            .arg("-I").arg(&include)
            .arg("-o").arg(&obj)
            .arg(&src)
            .status()
            .unwrap_or_else(|e| panic!("ffai-attn-sys: cannot run {nvcc}: {e}"));
        assert!(st.success(), "ffai-attn-sys: nvcc failed on {}", src.display());
        objs.push(obj);
    }
    let lib = out.join("libffai_attn.a");
    let _ = std::fs::remove_file(&lib);
    let st = Command::new("ar").arg("crs").arg(&lib).args(&objs).status()
        .expect("ffai-attn-sys: cannot run ar");
    assert!(st.success(), "ffai-attn-sys: ar failed");

    println!("cargo:rustc-link-search=native={}", out.display());
    println!("cargo:rustc-link-lib=static=ffai_attn");
    println!("cargo:rustc-link-search=native={}/lib64", cuda_home);
    println!("cargo:rustc-link-lib=static=cudart_static");
    for l in ["stdc++", "dl", "rt", "pthread"] {
        println!("cargo:rustc-link-lib=dylib={l}");
    }
}

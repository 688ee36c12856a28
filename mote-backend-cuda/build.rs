//! Builds `libmote_cuda` (the sm_100a kernels and the C ABI of
//! include/mote_cuda.h) into a static archive for the `cuda` feature -- the
//! shape of crates/mote-backend-hip/build.rs:40-92 with nvcc in place of
//! hipcc.
//!
//! The kernels are one CUDA translation unit (`csrc/libmote_cuda.cu`
//! includes the others), compiled for `sm_$MOTE_CUDA_ARCH` (default
//! `100a`: B200; sm_100a code runs only there).  `NVCC` and `AR` select
//! the tools, `MOTE_CUDA_SRC` the directory holding `csrc/` and `include/`
//! (default: the crate directory).  NCCL is opened with dlopen at first
//! use, so only cudart, libstdc++ and libdl are linked.
//!
//! NOT COMPILED HERE (no cargo in this environment).

fn main() {
    use std::{env, path::PathBuf, process::Command};

    println!("cargo:rerun-if-env-changed=MOTE_CUDA_ARCH");
    println!("cargo:rerun-if-env-changed=MOTE_CUDA_SRC");
    println!("cargo:rerun-if-env-changed=NVCC");
    println!("cargo:rerun-if-env-changed=AR");
    if env::var_os("CARGO_FEATURE_CUDA").is_none() {
        return;
    }

    let root = PathBuf::from(env::var("MOTE_CUDA_SRC").unwrap_or_else(|_| {
        env::var("CARGO_MANIFEST_DIR").expect("cargo sets CARGO_MANIFEST_DIR")
    }));
    let csrc = root.join("csrc");
    let include = root.join("include");
    println!("cargo:rerun-if-changed={}", csrc.display());
    println!("cargo:rerun-if-changed={}", include.display());

    let arch = env::var("MOTE_CUDA_ARCH").unwrap_or_else(|_| "100a".to_owned());
    let out_dir = PathBuf::from(env::var_os("OUT_DIR").expect("cargo sets OUT_DIR"));
    let object = out_dir.join("libmote_cuda.o");
    let archive = out_dir.join("libmote_cuda_kernels.a");

    let nvcc = env::var_os("NVCC").unwrap_or_else(|| "nvcc".into());
    let source = csrc.join("libmote_cuda.cu");
    let status = Command::new(&nvcc)
        .arg("-c")
        .arg(&source)
        .arg(format!("-gencode=arch=compute_{arch},code=sm_{arch}"))
        .args(["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC"])
        .arg("-I")
        .arg(&include)
        .arg("-o")
        .arg(&object)
        .status()
        .unwrap_or_else(|error| panic!("failed to spawn {nvcc:?} for {source:?}: {error}"));
    assert!(status.success(), "nvcc failed for {source:?} with sm_{arch}");

    // Rebuild the archive from scratch so no stale member survives.
    let _ = std::fs::remove_file(&archive);
    let ar = env::var_os("AR").unwrap_or_else(|| "ar".into());
    let status = Command::new(&ar)
        .arg("rcs")
        .arg(&archive)
        .arg(&object)
        .status()
        .unwrap_or_else(|error| panic!("failed to spawn {ar:?}: {error}"));
    assert!(status.success(), "ar failed for {archive:?}");

    println!("cargo:rustc-link-search=native={}", out_dir.display());
    println!("cargo:rustc-link-lib=static=mote_cuda_kernels");
    if let Some(cuda) = env::var_os("CUDA_HOME") {
        println!("cargo:rustc-link-search=native={}", PathBuf::from(cuda).join("lib64").display());
    }
    println!("cargo:rustc-link-lib=static=cudart_static");
    println!("cargo:rustc-link-lib=dylib=stdc++");
    println!("cargo:rustc-link-lib=dylib=dl");
    println!("cargo:rustc-link-lib=dylib=rt");
    println!("cargo:rustc-link-lib=dylib=pthread");
}

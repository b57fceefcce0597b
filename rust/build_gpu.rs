//! The nvcc step a Momiru build adds to its `build.rs` (reference build.rs
//! `main`, build.rs:217-276) to build and link the B200 matmul library when the
//! `gpu-gemm` feature is enabled: each CUDA unit of momiru_b200/csrc compiles
//! for sm_100a in parallel, nvcc links `libmomiru_gemm.so` into OUT_DIR, and
//! cargo links it with an rpath so the built crate finds it.
//!
//! `main` of build.rs calls `build_gpu_gemm()` after its existing directives.
//! NOT COMPILED HERE (no Rust toolchain in the build image); the same flags
//! are the ones momiru_b200/build.py uses.

use std::env;
use std::path::{Path, PathBuf};
use std::process::Command;

const UNITS: [&str; 5] = ["momiru_gemm", "tc_strict_pair", "tc_tf32_pair", "tc_strict_1cta", "tc_tf32_1cta"];
const FLAGS: [&str; 16] = [
    "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17", "-ftz=false",
    "-prec-div=true", "-prec-sqrt=true", "-fmad=true", "-Xcompiler", "-fPIC", "-Xcompiler",
    "-fvisibility=hidden", "--expt-relaxed-constexpr", "-Xcompiler", "-Wall",
];

fn nvcc() -> PathBuf {
    let home = env::var("CUDA_HOME").unwrap_or_else(|_| "/usr/local/cuda".to_owned());
    Path::new(&home).join("bin").join("nvcc")
}

pub fn build_gpu_gemm() {
    if env::var_os("CARGO_FEATURE_GPU_GEMM").is_none() {
        return;
    }
    println!("cargo:rerun-if-env-changed=CUDA_HOME");
    let root = PathBuf::from(env::var("CARGO_MANIFEST_DIR").expect("manifest dir"));
    let csrc = root.join("momiru_b200").join("csrc");
    println!("cargo:rerun-if-changed={}", csrc.display());
    println!("cargo:rerun-if-changed={}", root.join("include").join("momiru_gemm.h").display());
    let out = PathBuf::from(env::var("OUT_DIR").expect("out dir"));
    let objs: Vec<PathBuf> = UNITS.iter().map(|u| out.join(format!("{u}.o"))).collect();
    let children: Vec<_> = UNITS
        .iter()
        .zip(&objs)
        .map(|(u, o)| {
            Command::new(nvcc())
                .args(FLAGS)
                .arg("-c")
                .arg("-o")
                .arg(o)
                .arg(csrc.join(format!("{u}.cu")))
                .spawn()
                .expect("nvcc could not start (CUDA toolkit with sm_100a support required)")
        })
        .collect();
    for (mut child, unit) in children.into_iter().zip(UNITS) {
        let st = child.wait().expect("nvcc");
        assert!(st.success(), "nvcc failed on {unit}.cu");
    }
    let lib = out.join("libmomiru_gemm.so");
    let st = Command::new(nvcc())
        .args(["-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o"])
        .arg(&lib)
        .args(&objs)
        .status()
        .expect("nvcc link");
    assert!(st.success(), "linking libmomiru_gemm.so failed");
    println!("cargo:rustc-link-search=native={}", out.display());
    println!("cargo:rustc-link-lib=dylib=momiru_gemm");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", out.display());
}

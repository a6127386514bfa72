//! Compiles the hand-written CUDA sources of liblq8 for sm_100a with nvcc and links them
//! statically into the crate, with the CUDA runtime. NCCL is opened at run time by the
//! library (dlopen), so nothing links against it here.
//!
//! Environment:
//!   LQ8_CSRC   directory of the .cu sources (default: the repository's csrc next to this crate)
//!   LQ8_INCLUDE directory holding lq8.h (default: the repository's include/)
//!   CUDA_HOME  CUDA toolkit root (default /usr/local/cuda); nvcc from $CUDA_HOME/bin
use std::env;
use std::path::{Path, PathBuf};
use std::process::Command;

const SOURCES: &[&str] = &[
    "lq8_runtime.cu", "lq8_q8.cu", "lq8_gemv.cu", "lq8_gemm_tc.cu", "lq8_gemm_f16.cu", "lq8_attn_prefill.cu", "lq8_moe.cu",
    "lq8_comm.cu", "lq8_ops.cu", "lq8_attention.cu", "lq8_decode.cu", "lq8_sample.cu", "lq8_qwen3.cu",
];

fn main() {
    let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap());
    let repo = manifest.join("../..");
    let csrc = env::var("LQ8_CSRC").map(PathBuf::from).unwrap_or_else(|_| repo.join("qwen-omni-inference-rs_b200/csrc"));
    let include = env::var("LQ8_INCLUDE").map(PathBuf::from).unwrap_or_else(|_| repo.join("include"));
    let cuda = PathBuf::from(env::var("CUDA_HOME").unwrap_or_else(|_| "/usr/local/cuda".into()));
    let nvcc = cuda.join("bin/nvcc");
    let out = PathBuf::from(env::var("OUT_DIR").unwrap());

    let mut objects = Vec::new();
    for src in SOURCES {
        let input = csrc.join(src);
        let obj = out.join(Path::new(src).with_extension("o"));
        let status = Command::new(&nvcc)
            .args(["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17"])
            .args(["-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-I"])
            .arg(&include)
            .arg("-c")
            .arg(&input)
            .arg("-o")
            .arg(&obj)
            .status()
            .expect("failed to run nvcc (set CUDA_HOME)");
        assert!(status.success(), "nvcc failed on {}", input.display());
        println!("cargo:rerun-if-changed={}", input.display());
        objects.push(obj);
    }
    for hdr in ["lq8_internal.cuh", "lq8_fused.cuh", "lq8_async.cuh", "lq8_tma.cuh"] {
        println!("cargo:rerun-if-changed={}", csrc.join(hdr).display());
    }
    println!("cargo:rerun-if-changed={}", include.join("lq8.h").display());

    // each translation unit carries its own sm_100a image (no relocatable device code), as in
    // the repository's build.py; the archive is linked whole so every image registers
    let lib = out.join("liblq8.a");
    let _ = std::fs::remove_file(&lib);
    let status = Command::new("ar").arg("crs").arg(&lib).args(&objects).status().expect("ar");
    assert!(status.success(), "ar failed");

    println!("cargo:rustc-link-search=native={}", out.display());
    println!("cargo:rustc-link-lib=static:+whole-archive=lq8");
    println!("cargo:rustc-link-search=native={}", cuda.join("lib64").display());
    println!("cargo:rustc-link-lib=static=cudart_static");
    for l in ["dl", "rt", "pthread", "stdc++"] {
        println!("cargo:rustc-link-lib=dylib={l}");
    }
    println!("cargo:rerun-if-env-changed=LQ8_CSRC");
    println!("cargo:rerun-if-env-changed=LQ8_INCLUDE");
    println!("cargo:rerun-if-env-changed=CUDA_HOME");
}

//! Builds libcudabridge.so (sm_100a) with nvcc and links the crate against it.
//!
//! Inputs (environment):
//!   RUSTANE_B200_DIR  checkout of this repository (default: two levels above this crate)
//!   CUDA_HOME         CUDA 12.9 or newer (default /usr/local/cuda); nvcc cross-compiles
//!                     sm_100a without a GPU
//!   NCCL_HOME         NCCL install with include/nccl.h and lib/libnccl.so.2; only the
//!                     header is needed at build time (the library is opened with dlopen
//!                     when a tensor-parallel context is created; $CB_NCCL_LIB overrides
//!                     the path at run time)
//! The library is written to OUT_DIR and found at run time through an rpath entry.
use std::env;
use std::path::PathBuf;
use std::process::Command;

fn main() {
    let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap());
    let root = env::var("RUSTANE_B200_DIR")
        .map(PathBuf::from)
        .unwrap_or_else(|_| manifest.join("../.."));
    let cuda = PathBuf::from(env::var("CUDA_HOME").unwrap_or_else(|_| "/usr/local/cuda".into()));
    let nccl = env::var("NCCL_HOME")
        .map(PathBuf::from)
        .expect("NCCL_HOME must point at an NCCL install (include/nccl.h)");
    let out = PathBuf::from(env::var("OUT_DIR").unwrap());
    let lib = out.join("libcudabridge.so");
    let csrc = root.join("rustane_b200/csrc");
    let nccl_lib = nccl.join("lib/libnccl.so.2");

    let status = Command::new(cuda.join("bin/nvcc"))
        .args(["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17"])
        .args(["-Xcompiler", "-fPIC", "-shared", "--expt-relaxed-constexpr"])
        .arg(format!("-I{}", root.join("include").display()))
        .arg(format!("-I{}", csrc.display()))
        .arg(format!("-I{}", nccl.join("include").display()))
        .arg(format!("-DCB_NCCL_DEFAULT_PATH=\"{}\"", nccl_lib.display()))
        .arg("-o")
        .arg(&lib)
        .arg(csrc.join("bridge.cu"))
        .args(["-ldl", "-lpthread"])
        .status()
        .expect("failed to run nvcc");
    assert!(status.success(), "nvcc build of libcudabridge.so failed");

    println!("cargo:rustc-link-search=native={}", out.display());
    println!("cargo:rustc-link-lib=dylib=cudabridge");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", out.display());
    println!("cargo:rerun-if-changed={}", csrc.display());
    println!("cargo:rerun-if-changed={}", root.join("include/cuda_bridge.h").display());
    println!("cargo:rerun-if-env-changed=RUSTANE_B200_DIR");
    println!("cargo:rerun-if-env-changed=CUDA_HOME");
    println!("cargo:rerun-if-env-changed=NCCL_HOME");
}

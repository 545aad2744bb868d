//! Compiles libb200attn.so for sm_100a with nvcc from the package's CUDA sources
//! (`../../csrc`, headers in `../../../include`) and links it.  NVCC and CUDA_ARCH_FLAGS
//! may override the compiler and the -gencode flags.
use std::env;
use std::path::PathBuf;
use std::process::Command;

fn main() {
    let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap());
    let csrc = manifest.join("../../csrc");
    let include = manifest.join("../../../include");
    let out = PathBuf::from(env::var("OUT_DIR").unwrap());
    let nvcc = env::var("NVCC").unwrap_or_else(|_| "nvcc".to_string());
    let arch = env::var("CUDA_ARCH_FLAGS")
        .unwrap_or_else(|_| "-gencode arch=compute_100a,code=sm_100a".to_string());
    let sources = ["attn_fwd.cu", "block_ops.cu", "dequant.cu", "gemm.cu", "host_layout.cpp", "tp.cpp"];
    let mut cmd = Command::new(&nvcc);
    cmd.args(arch.split_whitespace())
        .args(["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "-shared",
               "-cudart", "static"])
        .arg(format!("-I{}", include.display()))
        .arg("-o")
        .arg(out.join("libb200attn.so"));
    for s in sources {
        cmd.arg(csrc.join(s));
        println!("cargo:rerun-if-changed={}", csrc.join(s).display());
    }
    cmd.arg("-ldl");
    let status = cmd.status().expect("failed to run nvcc (set NVCC to its path)");
    assert!(status.success(), "nvcc failed building libb200attn.so");
    println!("cargo:rerun-if-changed={}", csrc.join("ptx.cuh").display());
    println!("cargo:rerun-if-changed={}", include.display());
    println!("cargo:rerun-if-env-changed=NVCC");
    println!("cargo:rerun-if-env-changed=CUDA_ARCH_FLAGS");
    println!("cargo:rustc-link-search=native={}", out.display());
    println!("cargo:rustc-link-lib=dylib=b200attn");
    // let binaries find the library next to the build output without LD_LIBRARY_PATH
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", out.display());
}

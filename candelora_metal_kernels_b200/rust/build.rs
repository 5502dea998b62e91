//! Compiles the CUDA sources of libcandelora_iq2 (../csrc/*.cu) with nvcc for sm_100a into a static
//! library and links it with the CUDA runtime (static) and NCCL. The same flags as
//! candelora_metal_kernels_b200/build.py: -O3, -std=c++17, -gencode arch=compute_100a,code=sm_100a.
use std::env;
use std::path::{Path, PathBuf};
use std::process::Command;

const SOURCES: &[&str] = &[
    "iq2xxs_capi.cu",
    "iq2xxs_gemv.cu",
    "iq2xxs_gemm.cu",
    "iq2xxs_dequant.cu",
    "iq2xxs_noalloc.cu",
    "iq2xxs_sharded.cu",
    "iq2_variants.cu",
];

fn main() {
    let here = PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap());
    let csrc = here.join("..").join("csrc");
    let include = here.join("..").join("..").join("include");
    let out = PathBuf::from(env::var("OUT_DIR").unwrap());
    let cuda = env::var("CUDA_HOME").unwrap_or_else(|_| "/usr/local/cuda".to_string());
    let nvcc = Path::new(&cuda).join("bin").join("nvcc");

    let mut objs = Vec::new();
    for src in SOURCES {
        let obj = out.join(format!("{}.o", src.trim_end_matches(".cu")));
        let status = Command::new(&nvcc)
            .args(["-std=c++17", "-O3", "-lineinfo", "-gencode", "arch=compute_100a,code=sm_100a"])
            .args(["-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr"])
            .arg("-I").arg(&csrc)
            .arg("-I").arg(&include)
            .arg("-c").arg(csrc.join(src))
            .arg("-o").arg(&obj)
            .status()
            .expect("nvcc (set CUDA_HOME) must be installed to build the sm_100a kernels");
        assert!(status.success(), "nvcc failed on {src}");
        objs.push(obj);
        println!("cargo:rerun-if-changed={}", csrc.join(src).display());
    }
    let lib = out.join("libcandelora_iq2.a");
    let status = Command::new(&nvcc).arg("-lib").arg("-o").arg(&lib).args(&objs).status().unwrap();
    assert!(status.success(), "nvcc -lib failed");
    for h in ["iq2xxs_common.cuh", "iq2xxs_codebook.h", "iq2xxs_internal.h", "iq2_variant_grids.h"] {
        println!("cargo:rerun-if-changed={}", csrc.join(h).display());
    }
    println!("cargo:rerun-if-changed={}", include.join("candelora_iq2.h").display());
    println!("cargo:rustc-link-search=native={}", out.display());
    println!("cargo:rustc-link-search=native={}", Path::new(&cuda).join("lib64").display());
    println!("cargo:rustc-link-lib=static=candelora_iq2");
    println!("cargo:rustc-link-lib=static=cudart_static");
    println!("cargo:rustc-link-lib=dylib=nccl");
    println!("cargo:rustc-link-lib=dylib=stdc++");
    println!("cargo:rustc-link-lib=dylib=dl");
    println!("cargo:rustc-link-lib=dylib=rt");
    println!("cargo:rerun-if-env-changed=CUDA_HOME");
}

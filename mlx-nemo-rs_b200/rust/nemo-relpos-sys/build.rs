//! Compiles the library's CUDA and C++ sources (mlx-nemo-rs_b200/csrc) with
//! nvcc through `cc`, for sm_100a only, and links them statically with the
//! static CUDA runtime.  NCCL is opened with dlopen at run time (the
//! sequence split); only its header is needed here: NCCL_INCLUDE points at
//! the directory of nccl.h when it is not under CUDA_HOME/include.
use std::env;
use std::path::PathBuf;

const CUDA_SOURCES: &[&str] = &[
    "gemm_sm100.cu", "gemm_tf32.cu", "attn_sm100.cu", "attn_simt.cu", "attn_stream.cu",
    "kernels_misc.cu",
    "noalloc.cu", "block_kernels.cu", "subsampling_kernels.cu",
];
const CPP_SOURCES: &[&str] = &["api.cpp", "halo.cpp", "block.cpp", "subsampling.cpp"];

fn main() {
    let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap());
    // rust/nemo-relpos-sys -> mlx-nemo-rs_b200/csrc and the repository's include/
    let pkg = manifest.join("..").join("..");
    let csrc = pkg.join("csrc");
    let include = pkg.join("..").join("include");
    let cuda_home = env::var("CUDA_HOME").unwrap_or_else(|_| "/usr/local/cuda".into());
    let nccl_include = env::var("NCCL_INCLUDE").unwrap_or_else(|_| format!("{cuda_home}/include"));

    let mut b = cc::Build::new();
    b.cuda(true)
        .cudart("static")
        .flag("-gencode=arch=compute_100a,code=sm_100a")
        .flag("-std=c++17")
        .flag("-O3")
        .flag("-lineinfo")
        .flag("--expt-relaxed-constexpr")
        .include(&csrc)
        .include(&include)
        .include(&nccl_include);
    for f in CUDA_SOURCES.iter().chain(CPP_SOURCES) {
        let path = csrc.join(f);
        println!("cargo:rerun-if-changed={}", path.display());
        // the .cpp files hold host code only; nvcc compiles them as C++
        if f.ends_with(".cpp") {
            b.file(&path).flag_if_supported("-x=cu");
        } else {
            b.file(&path);
        }
    }
    println!("cargo:rerun-if-changed={}", include.join("nemo_relpos.h").display());
    b.compile("nemo_relpos");
    println!("cargo:rustc-link-search=native={cuda_home}/lib64");
    println!("cargo:rustc-link-lib=static=cudart_static");
    for lib in ["dl", "rt", "pthread", "stdc++"] {
        println!("cargo:rustc-link-lib=dylib={lib}");
    }
    // the CUDA driver API (tensor maps) through the runtime's driver entry points
    println!("cargo:rustc-link-lib=dylib=cuda");
}

//! Compiles the CUDA sources of libthq4 (token-horizon_b200/csrc/*.cu) with
//! nvcc for sm_100a into a static library and links it with the CUDA runtime.
//! `NVCC` / `CUDA_HOME` select the toolkit (default /usr/local/cuda).
use std::path::PathBuf;

fn main() {
    let here = PathBuf::from(std::env::var("CARGO_MANIFEST_DIR").unwrap());
    let csrc = here.join("../../csrc").canonicalize().expect("token-horizon_b200/csrc");
    let include = here.join("../../../include").canonicalize().expect("include/");
    let cuda = std::env::var("CUDA_HOME").unwrap_or_else(|_| "/usr/local/cuda".into());

    let mut sources: Vec<PathBuf> = std::fs::read_dir(&csrc)
        .unwrap()
        .filter_map(|e| e.ok().map(|e| e.path()))
        .filter(|p| p.extension().map_or(false, |x| x == "cu"))
        .collect();
    sources.sort();

    let mut b = cc::Build::new();
    b.cuda(true)
        .cudart("shared")
        .include(&include)
        .include(&csrc)
        .flag("-gencode")
        .flag("arch=compute_100a,code=sm_100a")
        .flag("-O3")
        .flag("-lineinfo")
        .flag("-std=c++17")
        .flag("--expt-relaxed-constexpr")
        .flag("-diag-suppress")
        .flag("177");
    for s in &sources {
        b.file(s);
        println!("cargo:rerun-if-changed={}", s.display());
    }
    for h in ["thq4_common.cuh", "thq4_internal.h"] {
        println!("cargo:rerun-if-changed={}", csrc.join(h).display());
    }
    println!("cargo:rerun-if-changed={}", include.join("thq4.h").display());
    b.compile("thq4");

    println!("cargo:rustc-link-search=native={cuda}/lib64");
    println!("cargo:rustc-link-lib=dylib=cudart");
    println!("cargo:rustc-link-lib=dylib=stdc++");
}

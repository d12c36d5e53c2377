// Compiles the library's .cu sources with nvcc for sm_100a into
// $OUT_DIR/libbmlattn.so and links it.  No Triton, no CPU fallback, no
// multi-backend dispatch: without the library or a GPU the calls return an
// error status.
use std::{env, path::PathBuf, process::Command};

fn main() {
    let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap());
    let root = env::var("BML_B200_DIR").map(PathBuf::from).unwrap_or_else(|_| manifest.join("../.."));
    let csrc = root.join("bml_b200/csrc");
    let out = PathBuf::from(env::var("OUT_DIR").unwrap());
    let mut srcs: Vec<PathBuf> = std::fs::read_dir(&csrc)
        .expect("bml_b200/csrc (set BML_B200_DIR)")
        .filter_map(|e| e.ok().map(|e| e.path()))
        .filter(|p| p.extension().map_or(false, |x| x == "cu"))
        .collect();
    srcs.sort();
    let nvcc = env::var("NVCC").unwrap_or_else(|_| "nvcc".into());
    let status = Command::new(nvcc)
        .args(["-std=c++17", "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
               "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared", "-o"])
        .arg(out.join("libbmlattn.so"))
        .args(&srcs)
        .status()
        .expect("nvcc");
    assert!(status.success(), "nvcc failed");
    println!("cargo:rustc-link-search=native={}", out.display());
    println!("cargo:rustc-link-lib=dylib=bmlattn");
    println!("cargo:rustc-link-lib=dylib=cudart");
    println!("cargo:rerun-if-changed={}", csrc.display());
    println!("cargo:rerun-if-changed={}", root.join("include").display());
    println!("cargo:rerun-if-env-changed=BML_B200_DIR");
}

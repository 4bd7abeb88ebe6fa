// Build hook of the CUDA backend.  It replaces nodestor-vulkan/build.rs:7-59,
// which compiles the GLSL shaders through naga: here `make` runs nvcc on the
// hand-written .cu files for sm_100a and links the resulting libnsq.so.
//
// NSQ_ROOT is the root of the libnsq source tree (the directory holding
// include/nsq.h and planejaja_b200/csrc).  CUDA_HOME defaults to
// /usr/local/cuda.
use std::env;
use std::path::PathBuf;
use std::process::Command;

fn main() {
    let root = PathBuf::from(env::var("NSQ_ROOT").expect("NSQ_ROOT: path of the libnsq source tree"));
    let csrc = root.join("planejaja_b200").join("csrc");
    let status = Command::new("make")
        .arg("-C")
        .arg(&csrc)
        .status()
        .expect("running make for libnsq");
    assert!(status.success(), "libnsq build failed");
    let cuda = env::var("CUDA_HOME").unwrap_or_else(|_| "/usr/local/cuda".to_string());
    println!("cargo:rustc-link-search=native={}", root.join("planejaja_b200").display());
    println!("cargo:rustc-link-search=native={cuda}/lib64");
    println!("cargo:rustc-link-lib=dylib=nsq");
    println!("cargo:rustc-link-lib=dylib=cudart");
    println!("cargo:rerun-if-changed={}", csrc.display());
    println!("cargo:rerun-if-changed={}", root.join("include").join("nsq.h").display());
    println!("cargo:rerun-if-env-changed=NSQ_ROOT");
}

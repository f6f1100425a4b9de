//! Links libqwen_cuda.so.  The library is built by `python qwen-30brust_b200/build.py` (nvcc,
//! sm_100a) next to its sources; QWEN_CUDA_LIB_DIR overrides where to look for it.
use std::{env, path::PathBuf};

fn main() {
    let dir = match env::var("QWEN_CUDA_LIB_DIR") {
        Ok(d) => PathBuf::from(d),
        Err(_) => PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap()).join("../../qwen-30brust_b200"),
    };
    if !dir.join("libqwen_cuda.so").exists() {
        println!(
            "cargo:warning=libqwen_cuda.so not found in {} (build it with qwen-30brust_b200/build.py or set QWEN_CUDA_LIB_DIR)",
            dir.display()
        );
    }
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=qwen_cuda");
    // the engine links the CUDA runtime statically; it still needs the driver at run time
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
    println!("cargo:rerun-if-env-changed=QWEN_CUDA_LIB_DIR");
    println!("cargo:rerun-if-changed=../../include/qwen_cuda.h");
}

//! Builds libllmhost_kv.so with nvcc (sm_100a) and links it.
//!
//! LLMHOST_B200_DIR   checkout of the library (default: two levels above this crate)
//! LLMHOST_KV_PREBUILT set to use the .so already under llmhost_b200/_lib
//! CUDA_HOME          toolkit root for the CUDA runtime (default /usr/local/cuda)

use std::{env, path::PathBuf, process::Command};

fn main() {
    let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").expect("cargo sets CARGO_MANIFEST_DIR"));
    let src = env::var_os("LLMHOST_B200_DIR")
        .map(PathBuf::from)
        .unwrap_or_else(|| manifest.join("..").join(".."));
    if env::var_os("LLMHOST_KV_PREBUILT").is_none() {
        let status = Command::new("python3")
            .args(["-m", "llmhost_b200.build"])
            .current_dir(&src)
            .status()
            .expect("run the nvcc build of libllmhost_kv (python3 -m llmhost_b200.build)");
        assert!(status.success(), "libllmhost_kv build failed");
    }
    let lib_dir = src.join("llmhost_b200").join("_lib");
    println!("cargo:rustc-link-search=native={}", lib_dir.display());
    println!("cargo:rustc-link-lib=dylib=llmhost_kv");
    // DeviceBuffer (Backend::alloc) calls the CUDA runtime directly.
    let cuda = env::var_os("CUDA_HOME").map(PathBuf::from).unwrap_or_else(|| PathBuf::from("/usr/local/cuda"));
    println!("cargo:rustc-link-search=native={}", cuda.join("lib64").display());
    println!("cargo:rustc-link-lib=dylib=cudart");
    println!("cargo:rerun-if-changed={}", src.join("include").join("llmhost_kv.h").display());
    println!("cargo:rerun-if-changed={}", src.join("llmhost_b200").join("csrc").display());
    println!("cargo:rerun-if-env-changed=LLMHOST_B200_DIR");
    println!("cargo:rerun-if-env-changed=LLMHOST_KV_PREBUILT");
}

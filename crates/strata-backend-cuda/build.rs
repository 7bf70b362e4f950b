//! Finds (or builds) `libstrata_cuda.so` and links it.
//!
//! * `STRATA_CUDA_LIB_DIR` — a directory holding a prebuilt `libstrata_cuda.so`;
//! * otherwise `STRATA_CUDA_SRC` — the source tree whose `strata-rs_b200/build.py`
//!   compiles every kernel with `nvcc -gencode arch=compute_100a,code=sm_100a`
//!   into `strata-rs_b200/libstrata_cuda.so`.
//!
//! There is no CPU build of this crate: without one of the two the build fails.

use std::env;
use std::path::{Path, PathBuf};
use std::process::Command;

fn main() {
    println!("cargo:rerun-if-env-changed=STRATA_CUDA_LIB_DIR");
    println!("cargo:rerun-if-env-changed=STRATA_CUDA_SRC");
    println!("cargo:rerun-if-env-changed=PYTHON");

    let dir = if let Ok(d) = env::var("STRATA_CUDA_LIB_DIR") {
        PathBuf::from(d)
    } else if let Ok(src) = env::var("STRATA_CUDA_SRC") {
        build_from(Path::new(&src))
    } else {
        panic!(
            "strata-backend-cuda: set STRATA_CUDA_LIB_DIR to a directory with libstrata_cuda.so, \
             or STRATA_CUDA_SRC to its source tree (needs nvcc for sm_100a)"
        );
    };
    let lib = dir.join("libstrata_cuda.so");
    assert!(lib.is_file(), "strata-backend-cuda: {} not found", lib.display());
    println!("cargo:rerun-if-changed={}", lib.display());
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=strata_cuda");
    // this crate's own tests and examples find the library without LD_LIBRARY_PATH
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
    println!("cargo:lib_dir={}", dir.display());
}

fn build_from(src: &Path) -> PathBuf {
    for h in ["include/strata_cuda.h", "include/strata_gguf.h"] {
        println!("cargo:rerun-if-changed={}", src.join(h).display());
    }
    let csrc = src.join("strata-rs_b200/csrc");
    println!("cargo:rerun-if-changed={}", csrc.display());
    let python = env::var("PYTHON").unwrap_or_else(|_| "python3".to_string());
    let status = Command::new(&python)
        .arg(src.join("strata-rs_b200/build.py"))
        .current_dir(src)
        .status()
        .unwrap_or_else(|e| panic!("strata-backend-cuda: cannot run {python}: {e}"));
    assert!(status.success(), "strata-backend-cuda: build.py failed ({status})");
    src.join("strata-rs_b200")
}

//! Link step for libheadshot_cuda.so.
//!
//! The library is built by `python -m headshot_b200.build` (nvcc, sm_100a)
//! into `headshot_b200/libheadshot_cuda.so` next to this crate; a host that
//! installs it elsewhere sets HEADSHOT_CUDA_LIB_DIR.  The CUDA runtime is
//! linked into the library itself, so nothing else is needed here; NCCL is
//! opened at run time by the library (multi-GPU calls only).
use std::env;
use std::path::PathBuf;

fn main() {
    println!("cargo:rerun-if-env-changed=HEADSHOT_CUDA_LIB_DIR");
    let dir = match env::var_os("HEADSHOT_CUDA_LIB_DIR") {
        Some(d) => PathBuf::from(d),
        None => PathBuf::from(env::var("CARGO_MANIFEST_DIR").expect("cargo sets CARGO_MANIFEST_DIR"))
            .join("..")
            .join("headshot_b200"),
    };
    println!("cargo:rerun-if-changed=../include/headshot_cuda.h");
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=headshot_cuda");
    // Let binaries of the workspace find the library at run time without LD_LIBRARY_PATH.
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
}

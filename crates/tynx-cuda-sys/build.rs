//! Link against the built engine: `python tynx_b200/build.py` writes
//! `tynx_b200/_lib/libtynx_cuda.so`; TYNX_CUDA_LIB_DIR overrides the directory.
use std::env;
use std::path::PathBuf;

fn main() {
    let dir = env::var("TYNX_CUDA_LIB_DIR").map(PathBuf::from).unwrap_or_else(|_| {
        PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap()).join("../../tynx_b200/_lib")
    });
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=tynx_cuda");
    println!("cargo:rerun-if-env-changed=TYNX_CUDA_LIB_DIR");
}

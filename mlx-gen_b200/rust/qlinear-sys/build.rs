//! Links libqlinear.so.  QLINEAR_LIB_DIR names the directory that holds it (the Python
//! package directory `mlx-gen_b200/qlinear` after `__graft_entry__.build()`); the CUDA
//! runtime and driver come in through the library's own DT_NEEDED entries.
use std::env;
use std::path::PathBuf;

fn main() {
    let dir = env::var("QLINEAR_LIB_DIR").map(PathBuf::from).unwrap_or_else(|_| {
        PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap()).join("../../qlinear")
    });
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=qlinear");
    println!("cargo:rerun-if-env-changed=QLINEAR_LIB_DIR");
    println!("cargo:rerun-if-changed=../../../include/qlinear.h");
}

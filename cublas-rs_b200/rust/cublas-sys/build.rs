// Builds libb2blas.so (nvcc, sm_100a) with the library's own Makefile and
// links it.  The library links the CUDA runtime statically and needs only
// the driver (libcuda.so) at run time.
use std::path::PathBuf;
use std::process::Command;

fn main() {
    let manifest = PathBuf::from(std::env::var("CARGO_MANIFEST_DIR").unwrap());
    // cublas-rs_b200/rust/cublas-sys -> cublas-rs_b200
    let pkg = manifest.join("../..").canonicalize().expect("cublas-rs_b200 directory");
    let st = Command::new("make").arg("-C").arg(&pkg).arg("-j").status().expect("running make");
    assert!(st.success(), "building libb2blas failed");
    let libdir = pkg.join("b2blas");
    println!("cargo:rustc-link-search=native={}", libdir.display());
    println!("cargo:rustc-link-lib=dylib=b2blas");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", libdir.display());
    println!("cargo:rerun-if-changed={}", pkg.join("csrc").display());
    println!("cargo:rerun-if-changed={}", pkg.join("../include/b2blas.h").display());
}

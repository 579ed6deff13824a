//! Builds libab2.so for sm_100a with the package's own build script (nvcc) and links the
//! crate against it. Set PYTHON to choose the interpreter (default python3).
use std::{env, path::PathBuf, process::Command};

fn main() {
    let crate_dir = PathBuf::from(env::var("CARGO_MANIFEST_DIR").expect("CARGO_MANIFEST_DIR"));
    let pkg = crate_dir.parent().expect("crate lives in ane-infer_b200/rust").to_path_buf();
    let include = pkg.parent().expect("repository root").join("include");
    let python = env::var("PYTHON").unwrap_or_else(|_| "python3".to_string());
    let status = Command::new(&python)
        .arg(pkg.join("build.py"))
        .status()
        .unwrap_or_else(|e| panic!("could not run {python} build.py: {e}"));
    assert!(status.success(), "libab2 build (nvcc, sm_100a) failed");
    println!("cargo:rustc-link-search=native={}", pkg.display());
    println!("cargo:rustc-link-lib=dylib=ab2");
    // this crate's own tests and examples find the library beside the sources
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", pkg.display());
    println!("cargo:rerun-if-changed={}", pkg.join("csrc").display());
    println!("cargo:rerun-if-changed={}", include.join("ab2.h").display());
    println!("cargo:rerun-if-env-changed=PYTHON");
}

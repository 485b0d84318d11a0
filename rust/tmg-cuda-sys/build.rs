//! Builds libtmg_cuda.so in the repository tree (nvcc, sm_100a) through the
//! Python build script, then tells cargo where to link it from.
//!
//! TMG_REPO overrides the repository root (default: two levels above this
//! crate); TMG_PYTHON the interpreter (default: python3).  TMG_SKIP_BUILD=1
//! links a library built beforehand without rebuilding it.
use std::env;
use std::path::PathBuf;
use std::process::Command;

fn main() {
    let crate_dir = PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap());
    let repo = env::var("TMG_REPO")
        .map(PathBuf::from)
        .unwrap_or_else(|_| crate_dir.join("..").join(".."));
    let python = env::var("TMG_PYTHON").unwrap_or_else(|_| "python3".to_string());
    if env::var("TMG_SKIP_BUILD").map(|v| v != "1").unwrap_or(true) {
        let status = Command::new(&python)
            .args(["-m", "tinyminigo_b200.build"])
            .current_dir(&repo)
            .status()
            .expect("could not run the Python build of libtmg_cuda.so");
        assert!(status.success(), "building libtmg_cuda.so failed");
    }
    let lib_dir = repo.join("tinyminigo_b200").join("lib");
    println!("cargo:rustc-link-search=native={}", lib_dir.display());
    println!("cargo:rustc-link-lib=dylib=tmg_cuda");
    // the engine finds the library next to the repository at run time
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", lib_dir.display());
    println!("cargo:rerun-if-changed={}", repo.join("include").join("tmg_cuda.h").display());
    println!("cargo:rerun-if-changed={}", repo.join("tinyminigo_b200").join("csrc").display());
    println!("cargo:rerun-if-env-changed=TMG_REPO");
    println!("cargo:rerun-if-env-changed=TMG_SKIP_BUILD");
}

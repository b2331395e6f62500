//! Links libfa_b200.so.  FA_B200_LIB_DIR names the directory that holds it
//! (default: ../lib, where `make -C flash-attention-cpu_b200` puts it).
use std::env;
use std::path::PathBuf;

fn main() {
    let dir = match env::var("FA_B200_LIB_DIR") {
        Ok(d) => PathBuf::from(d),
        Err(_) => PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap()).join("..").join("lib"),
    };
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=fa_b200");
    // found at run time without LD_LIBRARY_PATH
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
    println!("cargo:rerun-if-env-changed=FA_B200_LIB_DIR");
}

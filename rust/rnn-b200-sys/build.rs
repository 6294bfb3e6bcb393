// Links librnn_b200.so (built by `python -m rustnn_b200.build`).  The
// directory holding it comes from RNN_B200_LIB_DIR, else the `rustnn_b200`
// package directory of this repository; it is also added to the run-time
// search path so a binary finds the library without LD_LIBRARY_PATH.
use std::env;
use std::path::PathBuf;

fn main() {
    println!("cargo:rerun-if-env-changed=RNN_B200_LIB_DIR");
    let dir = match env::var("RNN_B200_LIB_DIR") {
        Ok(d) => PathBuf::from(d),
        Err(_) => PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap()).join("../../rustnn_b200"),
    };
    let dir = dir.canonicalize().unwrap_or(dir);
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=rnn_b200");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
    println!("cargo:rerun-if-changed={}", dir.join("librnn_b200.so").display());
}

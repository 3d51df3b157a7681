// Links libqora_mixer.so (built by `make -C qora-llm-4b_b200`).  The
// directory comes from QORA_MIXER_LIB_DIR, else the package directory two
// levels up, where the Makefile writes the library.
use std::env;
use std::path::PathBuf;

fn main() {
    let dir = env::var("QORA_MIXER_LIB_DIR").map(PathBuf::from).unwrap_or_else(|_| {
        PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap()).join("..").join("..")
    });
    println!("cargo:rerun-if-env-changed=QORA_MIXER_LIB_DIR");
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=qora_mixer");
}

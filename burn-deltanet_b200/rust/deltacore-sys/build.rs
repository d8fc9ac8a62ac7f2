// Not compiled here: no Rust toolchain in this image.
//
// Links libdeltacore.so.  DELTACORE_LIB_DIR names the directory that holds it (the package directory
// burn-deltanet_b200/ after `python burn-deltanet_b200/build.py`); the default is the crate's
// grandparent, which is that directory in this repository.
fn main() {
    let dir = std::env::var("DELTACORE_LIB_DIR").unwrap_or_else(|_| {
        let here = std::path::PathBuf::from(std::env::var("CARGO_MANIFEST_DIR").unwrap());
        here.join("../..").display().to_string()
    });
    println!("cargo:rerun-if-env-changed=DELTACORE_LIB_DIR");
    println!("cargo:rustc-link-search=native={dir}");
    println!("cargo:rustc-link-lib=dylib=deltacore");
}

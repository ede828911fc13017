// Links liblfm2_b200.so (built by lfm2-w9100-rust_b200/build.py). The
// directory comes from LFM2_B200_LIB_DIR, else the package directory two
// levels up from this crate, where build.py writes the library.
fn main() {
    let dir = std::env::var("LFM2_B200_LIB_DIR").unwrap_or_else(|_| {
        let here = std::path::PathBuf::from(std::env::var("CARGO_MANIFEST_DIR").unwrap());
        here.join("../..").canonicalize().unwrap().display().to_string()
    });
    println!("cargo:rustc-link-search=native={dir}");
    println!("cargo:rustc-link-lib=dylib=lfm2_b200");
    println!("cargo:rerun-if-env-changed=LFM2_B200_LIB_DIR");
}

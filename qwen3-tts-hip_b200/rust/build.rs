// Links libqtts_b200.so from the directory named by QTTS_B200_LIB_DIR
// (default: the package directory one level up, where `make` builds it).
fn main() {
    let dir = std::env::var("QTTS_B200_LIB_DIR").unwrap_or_else(|_| {
        let here = std::env::var("CARGO_MANIFEST_DIR").expect("CARGO_MANIFEST_DIR");
        format!("{here}/..")
    });
    println!("cargo:rustc-link-search=native={dir}");
    println!("cargo:rustc-link-lib=dylib=qtts_b200");
    println!("cargo:rerun-if-env-changed=QTTS_B200_LIB_DIR");
}

// Links libkyro_spec.so, built by `python -m kyro_b200.build`.  KYRO_SPEC_LIB_DIR
// names the directory that holds it (default: the kyro_b200 package beside
// this crate's repository).
fn main() {
    let dir = std::env::var("KYRO_SPEC_LIB_DIR").unwrap_or_else(|_| {
        let manifest = std::env::var("CARGO_MANIFEST_DIR").unwrap();
        format!("{manifest}/../../kyro_b200")
    });
    println!("cargo:rustc-link-search=native={dir}");
    println!("cargo:rustc-link-lib=dylib=kyro_spec");
    println!("cargo:rerun-if-env-changed=KYRO_SPEC_LIB_DIR");
}

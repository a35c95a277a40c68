// build.rs of the vestra-kernels crate, `b200` feature: links
// libvestra_b200.so (built by vestra-kernels_b200/build.py) from
// VESTRA_B200_LIB_DIR.  Not compiled in this repository (no Rust toolchain
// here); tests/test_rust_binding.py checks that src/b200/ffi.rs declares
// exactly the symbols of include/vestra_b200.h.
fn main() {
    if std::env::var_os("CARGO_FEATURE_B200").is_some() {
        let dir = std::env::var("VESTRA_B200_LIB_DIR").expect("VESTRA_B200_LIB_DIR");
        println!("cargo:rustc-link-search=native={dir}");
        println!("cargo:rustc-link-lib=dylib=vestra_b200");
        println!("cargo:rerun-if-env-changed=VESTRA_B200_LIB_DIR");
    }
}

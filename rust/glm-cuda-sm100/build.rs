// Links libglmaxx_sm100.so (python -m glmaxx_b200.build writes it next to the
// glmaxx_b200 package); the directory comes from GLMAXX_KERNEL_LIB_DIR, as for the
// reference's glmaxx_sm120 (crates/glm-cuda/build.rs:1-9).
fn main() {
    let dir = std::env::var("GLMAXX_KERNEL_LIB_DIR")
        .expect("GLMAXX_KERNEL_LIB_DIR must name the directory of libglmaxx_sm100.so");
    println!("cargo:rustc-link-search=native={dir}");
    println!("cargo:rustc-link-lib=dylib=glmaxx_sm100");
    println!("cargo:rerun-if-env-changed=GLMAXX_KERNEL_LIB_DIR");
}

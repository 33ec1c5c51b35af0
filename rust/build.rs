//! Links the prebuilt CUDA library (the CUDA runtime is statically inside it).
//! `ARCTIC_CUDA_LIB_DIR` names the folder of libarctic_cuda.so; by default the folder the
//! repository's `make -C snowflake-arctic-embed-s-rust_b200/csrc` writes it to.
fn main() {
    let dir = std::env::var("ARCTIC_CUDA_LIB_DIR").unwrap_or_else(|_| {
        let manifest = std::env::var("CARGO_MANIFEST_DIR").expect("cargo sets CARGO_MANIFEST_DIR");
        format!("{manifest}/../snowflake-arctic-embed-s-rust_b200/lib")
    });
    println!("cargo:rustc-link-search=native={dir}");
    println!("cargo:rustc-link-lib=dylib=arctic_cuda");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{dir}");
    println!("cargo:rerun-if-env-changed=ARCTIC_CUDA_LIB_DIR");
}

//! Links libhayai_cuda.so (built by `python -c "import __graft_entry__ as g; g.build()"`
//! in the hayai_b200 checkout).  HAYAI_CUDA_LIB_DIR points at its `hayai_b200/lib` folder.
//! The library links the CUDA runtime statically: only the NVIDIA driver is needed at run time.
fn main() {
    let dir = std::env::var("HAYAI_CUDA_LIB_DIR")
        .expect("set HAYAI_CUDA_LIB_DIR to the folder holding libhayai_cuda.so");
    println!("cargo:rustc-link-search=native={dir}");
    println!("cargo:rustc-link-lib=dylib=hayai_cuda");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{dir}");
    println!("cargo:rerun-if-env-changed=HAYAI_CUDA_LIB_DIR");
}

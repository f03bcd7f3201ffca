// Link libvmlm_cuda.so: its directory comes from VMLM_CUDA_LIB_DIR (the
// sparrow_b200/lib folder of a build of this repository).
fn main() {
    println!("cargo:rerun-if-env-changed=VMLM_CUDA_LIB_DIR");
    if let Ok(dir) = std::env::var("VMLM_CUDA_LIB_DIR") {
        println!("cargo:rustc-link-search=native={dir}");
    }
    println!("cargo:rustc-link-lib=dylib=vmlm_cuda");
}

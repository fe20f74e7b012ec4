// Cargo build script for the crate that includes `src/cuda`: links libssdllm_cuda.so,
// which `python ssd-llm_b200/build.py` compiles for sm_100a. SSDLLM_CUDA_DIR names the
// directory holding the library (default: ssd-llm_b200 beside the crate root).
fn main() {
    let dir = std::env::var("SSDLLM_CUDA_DIR").unwrap_or_else(|_| "ssd-llm_b200".into());
    println!("cargo:rustc-link-search=native={dir}");
    println!("cargo:rustc-link-lib=dylib=ssdllm_cuda");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{dir}");
    println!("cargo:rerun-if-changed={dir}/libssdllm_cuda.so");
    println!("cargo:rerun-if-env-changed=SSDLLM_CUDA_DIR");
}

//! B200 (sm_100a) compute backend for ssd-llm: the module a maintainer adds beside
//! `src/metal` (whose `mod.rs` declares `compute`, `gpu` and `neon`) and declares with
//! `mod cuda;` in `src/main.rs`. `ffi` binds `libssdllm_cuda.so` (the C ABI of
//! `include/ssdllm_cuda.h`); `compute` wraps it with `MetalCompute`'s method signatures.
pub mod compute;
pub mod ffi;

pub use compute::{CudaBatch, CudaCompute, CudaModel};

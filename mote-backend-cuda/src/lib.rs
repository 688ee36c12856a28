//! CUDA specialization backend: the hand-written sm_100a data plane for
//! mote's quantized linears and per-token layer kernels, behind the C ABI of
//! `include/mote_cuda.h` (`mote_cuda_*`, argument for argument the
//! `mote_hip_*` shims of crates/mote-backend-hip/src/ffi.rs plus this
//! backend's additions).
//!
//! * [`ffi`] declares every entry point;
//! * [`kernel`] registers them with `mote-kernel` as `KernelImpl`s keyed by
//!   operator, for `BackendKind::Cuda` devices, with the opaque-word
//!   argument convention;
//! * [`error`] maps status codes to `CudaError`.
//!
//! The typed, validating wrappers and the context/storage types follow the
//! HIP backend's (`HipContext`/`HipStorage` with the `hip` calls replaced);
//! their executable form is this repository's `mote_b200` Python package,
//! whose checks the GPU tests exercise.
//!
//! NOT COMPILED HERE: no cargo/rustc in the environment this repository is
//! built in.

#[cfg(feature = "cuda")]
pub mod error;
#[cfg(feature = "cuda")]
pub mod ffi;
#[cfg(feature = "cuda")]
pub mod kernel;

#[cfg(feature = "cuda")]
pub use error::CudaError;
#[cfg(feature = "cuda")]
pub use kernel::register;

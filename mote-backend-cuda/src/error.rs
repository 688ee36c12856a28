//! Status codes of the C ABI as a Rust error (the role of
//! crates/mote-backend-hip/src/error.rs:125-131 `check_hip`).
//!
//! NOT COMPILED HERE (no cargo in this environment).

use std::ffi::CStr;

use crate::ffi;

#[derive(Debug, thiserror::Error)]
pub enum CudaError {
    #[error("{operation} failed with status {status}: {message}")]
    Runtime {
        operation: &'static str,
        status: i32,
        message: String,
    },
}

/// Name of a status code (`mote_cuda_status_string`).
pub fn status_string(status: i32) -> String {
    // SAFETY: the library returns a static, NUL-terminated string.
    unsafe {
        let text = ffi::mote_cuda_status_string(status);
        if text.is_null() {
            format!("status {status}")
        } else {
            CStr::from_ptr(text).to_string_lossy().into_owned()
        }
    }
}

/// Non-zero status -> `CudaError::Runtime`.
pub fn check_cuda(status: i32, operation: &'static str) -> Result<(), CudaError> {
    if status == ffi::SUCCESS {
        Ok(())
    } else {
        Err(CudaError::Runtime {
            operation,
            status,
            message: status_string(status),
        })
    }
}

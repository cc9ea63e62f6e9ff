//! th-engine's Q4 affine quantized matmuls on B200 (sm_100a) for Rust.
//!
//! `ffi` declares the C ABI of libthq4 (include/thq4.h), which build.rs
//! compiles from token-horizon_b200/csrc with nvcc.  `check` turns a status
//! into an error carrying the library's message.  With the `candle` feature,
//! `candle_op` provides the CUDA counterparts of the engine's Metal custom
//! ops behind `QLin::linear_ps` and `QLin::gate_up_act_ps`
//! (engine/src/qwen35.rs:398, 711; engine/src/quant_kernel.rs:3040-3135).
pub mod ffi;

#[cfg(feature = "candle")]
pub mod candle_op;

use std::ffi::c_char;

/// A non-OK status with the message `thq4_last_error` held for this thread.
#[derive(Debug, Clone)]
pub struct Thq4Error {
    pub status: i32,
    pub message: String,
}

impl std::fmt::Display for Thq4Error {
    fn fmt(&self, f: &mut std::fmt::Formatter<'_>) -> std::fmt::Result {
        write!(f, "thq4 status {}: {}", self.status, self.message)
    }
}

impl std::error::Error for Thq4Error {}

/// `Ok(())` for THQ4_OK, else the status and the library's message.
pub fn check(status: ffi::thq4_status) -> Result<(), Thq4Error> {
    if status == ffi::THQ4_OK {
        return Ok(());
    }
    let mut buf = vec![0u8; 1024];
    let n = unsafe { ffi::thq4_last_error(buf.as_mut_ptr() as *mut c_char, buf.len()) }.min(buf.len() - 1);
    Err(Thq4Error { status, message: String::from_utf8_lossy(&buf[..n]).into_owned() })
}

/// "thq4 <semver> sm_100a".
pub fn version() -> String {
    unsafe { std::ffi::CStr::from_ptr(ffi::thq4_version()) }.to_string_lossy().into_owned()
}

/// Frag-layout buffer sizes (nibbles, scale/bias quads) for `rows` x `inp`.
pub fn weight_bytes(rows: i32, inp: i32) -> (usize, usize) {
    let (mut q, mut s) = (0usize, 0usize);
    unsafe { ffi::thq4_weight_bytes(rows, inp, 64, &mut q, &mut s) };
    (q, s)
}

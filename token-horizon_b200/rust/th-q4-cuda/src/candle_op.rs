//! candle CUDA custom ops for the engine's `QLin` (the counterparts of the
//! Metal ops in engine/src/quant_kernel.rs).
//!
//! The engine keeps each projection packed once at load (`QLin::tiled`,
//! engine/src/qwen35.rs:629-697); a CUDA build repacks into this library's
//! frag layout instead (`thq4_repack`) and keeps the two device buffers plus
//! a `thq4_weight` descriptor.  The ops below take (qw: U8 frag nibbles,
//! sb: BF16 or F16 scale/bias quads, x: BF16 [rows, in]) like the Metal ops
//! take (wq, sb, x), check their arguments before anything is launched
//! (check3, quant_kernel.rs:2671-2684), and return a fresh output buffer
//! that never aliases an input (quant_kernel.rs:3131).  Rows route as
//! `QLin::linear_ps` does (qwen35.rs:398-617): the library picks the decode
//! GEMV, the verify kernel or the prefill GEMM from the row count.
//!
//! Written against candle-core 0.11's CUDA backend (cudarc with explicit
//! streams); this image has no Rust toolchain, so it was not compiled here.
use std::ffi::c_void;
use std::sync::Mutex;

use candle_core::backend::BackendStorage;
use candle_core::cuda_backend::cudarc::driver::{CudaSlice, DevicePtr};
use candle_core::cuda_backend::WrapErr;
use candle_core::{CpuStorage, CudaStorage, CustomOp3, DType, Layout, Result, Shape};

use crate::ffi;

fn thq4(status: ffi::thq4_status) -> Result<()> {
    crate::check(status).map_err(candle_core::Error::wrap)
}

fn contiguous(l: &Layout, what: &str) -> Result<usize> {
    match l.contiguous_offsets() {
        Some((start, _)) => Ok(start),
        None => candle_core::bail!("thq4: {what} must be contiguous"),
    }
}

/// A zero-filled workspace per device, grown as needed and reused by every
/// later call on that device (each completed call leaves its counters zero).
/// Calls are stream-ordered on the device's one stream, as candle issues them.
static WORKSPACES: Mutex<Vec<(usize, CudaSlice<u8>)>> = Mutex::new(Vec::new());

fn with_workspace<R>(dev: &candle_core::CudaDevice, bytes: usize,
                     f: impl FnOnce(*mut c_void, usize) -> Result<R>) -> Result<R> {
    let mut all = WORKSPACES.lock().unwrap();
    let ord = dev.ordinal();
    let have = all.iter().position(|(o, s)| *o == ord && s.len() >= bytes);
    let idx = match have {
        Some(i) => i,
        None => {
            all.retain(|(o, _)| *o != ord);
            let ws = dev.alloc_zeros::<u8>(bytes.max(256)).w()?;
            all.push((ord, ws));
            all.len() - 1
        }
    };
    let stream = dev.cuda_stream();
    let (ptr, _guard) = all[idx].1.device_ptr(&stream);
    f(ptr as *mut c_void, all[idx].1.len())
}

/// `QLin::linear_ps` on CUDA: y [rows, out] bf16 = x [rows, in] bf16 . W^T.
pub struct Q4Linear {
    pub out: usize,
    pub inp: usize,
    /// THQ4_BF16 (the reference's scale format) or THQ4_F16
    pub sb_dtype: i32,
}

/// `QLin::gate_up_act_ps` on CUDA: y [rows, half] = bf16(silu(bf16 g) * bf16 u)
/// of a fused [gate | up] weight whose halves were packed separately
/// (`gate` holds rows [0, half), `up` rows [half, 2 half)).
pub struct Q4GateUp {
    pub half: usize,
    pub inp: usize,
    pub sb_dtype: i32,
    pub up_qw: usize,  // device address of the up half's nibbles
    pub up_sb: usize,  // device address of the up half's scale/bias quads
}

fn weight_desc(out: usize, inp: usize, sb_dtype: i32, qw: u64, sb: u64) -> Result<ffi::thq4_weight> {
    let mut w = ffi::thq4_weight { out: 0, inp: 0, gs: 0, sb_dtype: 0, qw: std::ptr::null(), sb: std::ptr::null() };
    thq4(unsafe {
        ffi::thq4_weight_init(&mut w, out as i32, inp as i32, 64, sb_dtype, qw as *const c_void, sb as *const c_void)
    })?;
    Ok(w)
}

fn rows_of(l_x: &Layout, inp: usize, who: &str) -> Result<usize> {
    let n = l_x.shape().elem_count();
    if inp % 64 != 0 || n % inp != 0 {
        candle_core::bail!("{who}: x {:?} vs in {inp} (want rows of a multiple of 64)", l_x.shape());
    }
    // activations are read as 16-byte vectors (qwen35.rs:7034-7037)
    if contiguous(l_x, "x")? % 8 != 0 {
        candle_core::bail!("{who}: x offset not 16-byte aligned");
    }
    Ok(n / inp)
}

fn out_shape(l_x: &Layout, cols: usize) -> Shape {
    let mut dims = l_x.shape().dims().to_vec();
    *dims.last_mut().unwrap() = cols;
    Shape::from(dims)
}

impl CustomOp3 for Q4Linear {
    fn name(&self) -> &'static str {
        "thq4-linear"
    }

    fn cpu_fwd(&self, _: &CpuStorage, _: &Layout, _: &CpuStorage, _: &Layout, _: &CpuStorage, _: &Layout)
               -> Result<(CpuStorage, Shape)> {
        candle_core::bail!("thq4-linear: CUDA only")
    }

    fn cuda_fwd(&self, s_qw: &CudaStorage, l_qw: &Layout, s_sb: &CudaStorage, l_sb: &Layout, s_x: &CudaStorage,
                l_x: &Layout) -> Result<(CudaStorage, Shape)> {
        if s_qw.dtype() != DType::U8 || s_x.dtype() != DType::BF16 {
            candle_core::bail!("thq4-linear: want qw u8 and x bf16");
        }
        let rows = rows_of(l_x, self.inp, "thq4-linear")?;
        let dev = s_x.device().clone();
        let stream = dev.cuda_stream();
        let qw = s_qw.as_cuda_slice::<u8>()?.slice(contiguous(l_qw, "qw")?..);
        let (qw_ptr, _g0) = qw.device_ptr(&stream);
        let sb_off = contiguous(l_sb, "sb")?;
        let (sb_ptr, _g1) = match s_sb.dtype() {
            DType::BF16 => s_sb.as_cuda_slice::<half::bf16>()?.slice(sb_off..).device_ptr(&stream),
            DType::F16 => s_sb.as_cuda_slice::<half::f16>()?.slice(sb_off..).device_ptr(&stream),
            _ => candle_core::bail!("thq4-linear: sb must be bf16 or f16"),
        };
        let w = weight_desc(self.out, self.inp, self.sb_dtype, qw_ptr, sb_ptr)?;
        let x = s_x.as_cuda_slice::<half::bf16>()?.slice(contiguous(l_x, "x")?..);
        let (x_ptr, _g2) = x.device_ptr(&stream);
        // a fresh output buffer, never a clone of an input's
        let y = unsafe { dev.alloc::<half::bf16>(rows * self.out) }.w()?;
        let (y_ptr, _g3) = y.device_ptr(&stream);
        let need = unsafe { ffi::thq4_linear_workspace_bytes(&w, rows as i32) };
        with_workspace(&dev, need, |ws, ws_bytes| {
            thq4(unsafe {
                ffi::thq4_linear(&w, x_ptr as *const c_void, ffi::THQ4_BF16, rows as i32, y_ptr as *mut c_void,
                                 ffi::THQ4_BF16, ws, ws_bytes, stream.cu_stream() as *mut c_void)
            })
        })?;
        drop((_g0, _g1, _g2, _g3));
        Ok((CudaStorage::wrap_cuda_slice(y, dev), out_shape(l_x, self.out)))
    }
}

impl CustomOp3 for Q4GateUp {
    fn name(&self) -> &'static str {
        "thq4-gate-up"
    }

    fn cpu_fwd(&self, _: &CpuStorage, _: &Layout, _: &CpuStorage, _: &Layout, _: &CpuStorage, _: &Layout)
               -> Result<(CpuStorage, Shape)> {
        candle_core::bail!("thq4-gate-up: CUDA only")
    }

    fn cuda_fwd(&self, s_qw: &CudaStorage, l_qw: &Layout, s_sb: &CudaStorage, l_sb: &Layout, s_x: &CudaStorage,
                l_x: &Layout) -> Result<(CudaStorage, Shape)> {
        if s_qw.dtype() != DType::U8 || s_x.dtype() != DType::BF16 {
            candle_core::bail!("thq4-gate-up: want qw u8 and x bf16");
        }
        let rows = rows_of(l_x, self.inp, "thq4-gate-up")?;
        let dev = s_x.device().clone();
        let stream = dev.cuda_stream();
        let qw = s_qw.as_cuda_slice::<u8>()?.slice(contiguous(l_qw, "qw")?..);
        let (qw_ptr, _g0) = qw.device_ptr(&stream);
        let sb_off = contiguous(l_sb, "sb")?;
        let (sb_ptr, _g1) = match s_sb.dtype() {
            DType::BF16 => s_sb.as_cuda_slice::<half::bf16>()?.slice(sb_off..).device_ptr(&stream),
            DType::F16 => s_sb.as_cuda_slice::<half::f16>()?.slice(sb_off..).device_ptr(&stream),
            _ => candle_core::bail!("thq4-gate-up: sb must be bf16 or f16"),
        };
        let gate = weight_desc(self.half, self.inp, self.sb_dtype, qw_ptr, sb_ptr)?;
        let up = weight_desc(self.half, self.inp, self.sb_dtype, self.up_qw as u64, self.up_sb as u64)?;
        let x = s_x.as_cuda_slice::<half::bf16>()?.slice(contiguous(l_x, "x")?..);
        let (x_ptr, _g2) = x.device_ptr(&stream);
        let y = unsafe { dev.alloc::<half::bf16>(rows * self.half) }.w()?;
        let (y_ptr, _g3) = y.device_ptr(&stream);
        let need = unsafe { ffi::thq4_linear_workspace_bytes(&gate, rows as i32) };
        with_workspace(&dev, need, |ws, ws_bytes| {
            thq4(unsafe {
                ffi::thq4_gate_up(&gate, &up, x_ptr as *const c_void, ffi::THQ4_BF16, rows as i32,
                                  y_ptr as *mut c_void, ffi::THQ4_BF16, ws, ws_bytes,
                                  stream.cu_stream() as *mut c_void)
            })
        })?;
        drop((_g0, _g1, _g2, _g3));
        Ok((CudaStorage::wrap_cuda_slice(y, dev), out_shape(l_x, self.half)))
    }
}

//! The C ABI of libthq4 (include/thq4.h), one declaration per entry point.
//! Pointers are device pointers unless the header says otherwise; `stream`
//! is a `cudaStream_t`; every call returns a `thq4_status` (0 = OK).
#![allow(non_camel_case_types)]
use std::ffi::{c_char, c_void};

pub type thq4_status = i32;
pub const THQ4_OK: thq4_status = 0;
pub const THQ4_ERR_INVALID_ARGUMENT: thq4_status = 1;
pub const THQ4_ERR_UNSUPPORTED: thq4_status = 2;
pub const THQ4_ERR_WORKSPACE: thq4_status = 3;
pub const THQ4_ERR_CUDA: thq4_status = 4;
pub const THQ4_ERR_NCCL: thq4_status = 5;

pub const THQ4_BF16: i32 = 0;
pub const THQ4_F16: i32 = 1;
pub const THQ4_F32: i32 = 2;

pub const THQ4_SRC_MLX: i32 = 0;
pub const THQ4_SRC_TILED: i32 = 1;
pub const THQ4_SRC_SLAB: i32 = 2;
pub const THQ4_SRC_FRAG: i32 = 3;

pub const THQ4_IPC_HANDLE_BYTES: usize = 64;

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct thq4_weight {
    pub out: i32,
    pub inp: i32,
    pub gs: i32,
    pub sb_dtype: i32,
    pub qw: *const c_void,
    pub sb: *const c_void,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct thq4_experts {
    pub experts: i32,
    pub out: i32,
    pub inp: i32,
    pub gs: i32,
    pub sb_dtype: i32,
    pub reserved: i32,
    pub qw: *const c_void,
    pub sb: *const c_void,
    pub qw_stride: u64,
    pub sb_stride: u64,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct thq4_q8_weight {
    pub out: i32,
    pub inp: i32,
    pub q: *const c_void,
    pub scales: *const c_void,
    pub biases: *const c_void,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct thq4_moe_weights {
    pub router: thq4_q8_weight,
    pub gate: thq4_experts,
    pub up: thq4_experts,
    pub down: thq4_experts,
    pub shared_gate: thq4_experts,
    pub shared_up: thq4_experts,
    pub shared_down: thq4_experts,
    pub shared_expert_gate: thq4_q8_weight,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct thq4_peer_gather {
    pub world: i32,
    pub rank: i32,
    pub rows: i32,
    pub offset: i32,
    pub stride: i32,
    pub wait: i32,
    pub dst: *const *mut c_void,
    pub flags: *const *mut u32,
    pub count: *mut u32,
    pub arrive: *mut u32,
    pub out_mode: i32,
    pub x_parts: i32,
    pub slot: i64,
    pub x_slot: i64,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct thq4_chain_op {
    pub w: *const thq4_weight,
    pub up: *const thq4_weight,
    pub x: *const c_void,
    pub y: *mut c_void,
    pub y_dtype: i32,
    pub reserved: i32,
}

extern "C" {
    pub fn thq4_version() -> *const c_char;
    pub fn thq4_last_error(buf: *mut c_char, cap: usize) -> usize;
    pub fn thq4_device_status(status_out: *mut u32, stream: *mut c_void) -> thq4_status;

    pub fn thq4_weight_bytes(rows: i32, inp: i32, gs: i32, qw_bytes: *mut usize, sb_bytes: *mut usize) -> usize;
    pub fn thq4_repack(src_layout: i32, src_w: *const c_void, src_sb: *const c_void, src_out: i32, inp: i32,
                       gs: i32, sb_dtype: i32, row_begin: i32, rows: i32, dst_qw: *mut c_void,
                       dst_qw_bytes: usize, dst_sb: *mut c_void, dst_sb_bytes: usize,
                       stream: *mut c_void) -> thq4_status;
    pub fn thq4_weight_init(w: *mut thq4_weight, out: i32, inp: i32, gs: i32, sb_dtype: i32, qw: *const c_void,
                            sb: *const c_void) -> thq4_status;

    pub fn thq4_linear(w: *const thq4_weight, x: *const c_void, x_dtype: i32, m: i32, y: *mut c_void,
                       y_dtype: i32, workspace: *mut c_void, workspace_bytes: usize,
                       stream: *mut c_void) -> thq4_status;
    pub fn thq4_gate_up(gate: *const thq4_weight, up: *const thq4_weight, x: *const c_void, x_dtype: i32, m: i32,
                        y: *mut c_void, y_dtype: i32, workspace: *mut c_void, workspace_bytes: usize,
                        stream: *mut c_void) -> thq4_status;
    pub fn thq4_linear_workspace_bytes(w: *const thq4_weight, m: i32) -> usize;
    pub fn thq4_linear_chain_workspace_bytes(ops: *const thq4_chain_op, n: i32) -> usize;
    pub fn thq4_linear_chain(ops: *const thq4_chain_op, n: i32, x_dtype: i32, m: i32, workspace: *mut c_void,
                             workspace_bytes: usize, stream: *mut c_void) -> thq4_status;
    pub fn thq4_linear_scalar(w: *const thq4_weight, x: *const c_void, x_dtype: i32, m: i32, y: *mut c_void,
                              y_dtype: i32, stream: *mut c_void) -> thq4_status;
    pub fn thq4_linear_noalloc(w: *const thq4_weight, x: *const c_void, x_dtype: i32, m: i32, y: *mut c_void,
                               y_dtype: i32, stream: *mut c_void) -> thq4_status;
    pub fn thq4_dequant(w: *const thq4_weight, y: *mut c_void, stream: *mut c_void) -> thq4_status;

    pub fn thq4_moe_max_tiles(t: i32, e: i32, k: i32) -> u32;
    pub fn thq4_moe_route(logits: *const c_void, t: i32, e: i32, k: i32, ids: *mut u32, weights: *mut c_void,
                          tiles: *mut u32, grouped_routes: *mut u32, route_rows: *mut u32, ntiles: *mut u32,
                          max_tiles: i32, stream: *mut c_void) -> thq4_status;
    pub fn thq4_moe_workspace_bytes(t: i32, h: i32, i: i32, e: i32, k: i32) -> usize;
    pub fn thq4_moe(x: *const c_void, residual: *const c_void, logits: *const c_void, t: i32, h: i32, i: i32,
                    e: i32, k: i32, gate: *const thq4_experts, up: *const thq4_experts, down: *const thq4_experts,
                    y: *mut c_void, workspace: *mut c_void, workspace_bytes: usize,
                    stream: *mut c_void) -> thq4_status;
    pub fn thq4_moe_scores_workspace_bytes(t: i32, ncols: i32) -> usize;
    pub fn thq4_moe_scores_q8(x: *const c_void, t: i32, router: *const thq4_q8_weight, ncols: i32,
                              scores: *mut c_void, ld: i32, workspace: *mut c_void, workspace_bytes: usize,
                              stream: *mut c_void) -> thq4_status;
    pub fn thq4_moe_add_max_tiles(t: i32, e: i32, k: i32, shared: i32) -> u32;
    pub fn thq4_moe_route_q8(x: *const c_void, t: i32, e: i32, k: i32, router: *const thq4_q8_weight,
                             shared_expert_gate: *const thq4_q8_weight, ids: *mut u32, weights: *mut c_void,
                             tiles: *mut u32, grouped_routes: *mut u32, route_rows: *mut u32, ntiles: *mut u32,
                             max_tiles: i32, workspace: *mut c_void, workspace_bytes: usize,
                             stream: *mut c_void) -> thq4_status;
    pub fn thq4_moe_add_workspace_bytes(t: i32, h: i32, i: i32, e: i32, k: i32, shared: i32) -> usize;
    pub fn thq4_moe_add(x: *const c_void, residual: *const c_void, t: i32, h: i32, i: i32, e: i32, k: i32,
                        w: *const thq4_moe_weights, y: *mut c_void, workspace: *mut c_void,
                        workspace_bytes: usize, stream: *mut c_void) -> thq4_status;

    pub fn thq4_linear_peer(w: *const thq4_weight, up: *const thq4_weight, x: *const c_void, x_dtype: i32, m: i32,
                            y: *mut c_void, workspace: *mut c_void, workspace_bytes: usize,
                            g: *const thq4_peer_gather, stream: *mut c_void) -> thq4_status;
    pub fn thq4_peer_wait(g: *const thq4_peer_gather, stream: *mut c_void) -> thq4_status;
    pub fn thq4_moe_partial(x: *const c_void, residual: *const c_void, logits: *const c_void, t: i32, h: i32,
                            i: i32, e: i32, k: i32, e0: i32, e1: i32, gate: *const thq4_experts,
                            up: *const thq4_experts, down: *const thq4_experts, y_part: *mut f32,
                            workspace: *mut c_void, workspace_bytes: usize, stream: *mut c_void) -> thq4_status;
    pub fn thq4_moe_add_partial_workspace_bytes(t: i32, h: i32, i: i32, e: i32, k: i32, e0: i32, e1: i32,
                                                shared_route: i32, runs_shared: i32) -> usize;
    pub fn thq4_moe_add_partial(x: *const c_void, residual: *const c_void, t: i32, h: i32, i: i32, e: i32, k: i32,
                                e0: i32, e1: i32, w: *const thq4_moe_weights, y_part: *mut f32,
                                workspace: *mut c_void, workspace_bytes: usize,
                                stream: *mut c_void) -> thq4_status;
    pub fn thq4_ipc_alloc(bytes: usize, ptr: *mut *mut c_void, handle: *mut c_void) -> thq4_status;
    pub fn thq4_ipc_open(handle: *const c_void, ptr: *mut *mut c_void) -> thq4_status;
    pub fn thq4_ipc_close(ptr: *mut c_void) -> thq4_status;
    pub fn thq4_ipc_free(ptr: *mut c_void) -> thq4_status;
    pub fn thq4_copy(dst: *mut c_void, src: *const c_void, bytes: usize, stream: *mut c_void) -> thq4_status;

    pub fn thq4_debug_set_gemv(chunk: i32, stages: i32, grid: i32, reserved: i32) -> thq4_status;
    pub fn thq4_debug_set_trace(buf: *mut c_void, bytes: usize) -> thq4_status;
    pub fn thq4_debug_gemv_plan(out: i32, inp: i32, m: i32, x_f32: i32, gate_up: i32, sms: i32,
                                cluster_fit: *const i32, plan: *mut i64) -> thq4_status;
    pub fn thq4_debug_prefill_plan(out: i32, inp: i32, m: i32, gate_up: i32, sms: i32, plan: *mut i64)
                                   -> thq4_status;
}

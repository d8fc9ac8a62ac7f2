//! Raw FFI of the B200 delta-rule core: `#[repr(C)]` mirrors of `include/deltacore.h`.
//!
//! Not compiled here: no Rust toolchain in this image.  The field order and C types of every struct are
//! checked against the header by `tests/test_rust_binding.py`, and every function declared below against
//! the symbols `libdeltacore.so` exports.
//!
//! Every pointer is a device pointer of the device current on the calling thread (host pointers for
//! `dc_chunk_fwd_host`); the caller owns every buffer and the library allocates nothing.  Calls enqueue on
//! `stream` and return a `dc_status`; the reference panics where these return an error, and [`check`]
//! restores that behaviour.
#![allow(non_camel_case_types)]

use std::ffi::{c_char, c_int, c_void, CStr};

/// `cudaStream_t` / `CUstream` (null = the legacy default stream).
pub type dc_stream_t = *mut c_void;

pub const DC_OK: c_int = 0;
pub const DC_EINVAL_SHAPE: c_int = 1;
pub const DC_EINVAL_WIDTH: c_int = 2;
pub const DC_EUNSUPPORTED_DTYPE: c_int = 3;
pub const DC_EINVAL_ARG: c_int = 4;
pub const DC_EUNSUPPORTED: c_int = 5;
pub const DC_ECUDA: c_int = 6;
pub const DC_EDEVICE: c_int = 7;
pub const DC_EWORKSPACE: c_int = 8;
pub const DC_ESCRATCH: c_int = 9;

pub const DC_F32: i32 = 0;
pub const DC_BF16: i32 = 1;

pub const DC_FLAG_FORCE_SIMT: u32 = 0x1;
pub const DC_FLAG_RECURRENT: u32 = 0x2;
pub const DC_FLAG_FORCE_SPLIT: u32 = 0x4;
/// Test hook of the failure path (the kernel issues no tile loads and its bounded waits run out).
pub const DC_FLAG_TEST_STALL: u32 = 0x100;

pub const DC_NOALLOC_SCRATCH_BYTES: u64 = 64 << 20;

pub const DC_PROLOGUE_CONV_SILU: u32 = 0x1;
pub const DC_PROLOGUE_QK_SILU: u32 = 0x2;
pub const DC_PROLOGUE_L2: u32 = 0x4;

pub const DC_GATE_WRITE: i32 = 0;
pub const DC_GATE_HEAD_DECAY: i32 = 1;
pub const DC_GATE_CHANNEL_DECAY: i32 = 2;

/// The prefill's arguments: `delta_chunk_recalculated`'s list
/// (src/delta/chunk_recalculated/chunk_recalculated.rs:115-126) as pointers plus shapes.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct dc_chunk_args {
    pub batch: i64,
    pub seq: i64,
    pub heads: i64,
    pub dk: i64,
    pub dv: i64,
    pub n_householder: i32,
    pub erase_w: i32,
    pub write_w: i32,
    pub g_w: i32,
    pub chunk_len: i32,
    pub in_dtype: i32,
    pub gate_dtype: i32,
    pub out_dtype: i32,
    pub flags: u32,
    pub scale: f64,
    pub q: *const c_void,
    pub k: *const c_void,
    pub v: *const c_void,
    pub erase: *const c_void,
    pub write: *const c_void,
    pub g: *const c_void,
    pub state_in: *const f32,
    pub y: *mut c_void,
    pub state_out: *mut f32,
    pub workspace: *mut c_void,
    pub workspace_bytes: u64,
}

/// One decode token: `delta_step`'s list (src/delta/recurrent.rs:41-50).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct dc_step_args {
    pub batch: i64,
    pub heads: i64,
    pub dk: i64,
    pub dv: i64,
    pub n_householder: i32,
    pub erase_w: i32,
    pub write_w: i32,
    pub g_w: i32,
    pub in_dtype: i32,
    pub gate_dtype: i32,
    pub out_dtype: i32,
    pub flags: u32,
    pub scale: f64,
    pub q: *const c_void,
    pub k: *const c_void,
    pub v: *const c_void,
    pub erase: *const c_void,
    pub write: *const c_void,
    pub g: *const c_void,
    pub state_in: *const f32,
    pub y: *mut c_void,
    pub state_out: *mut f32,
}

/// The backward (`combined_backward`, src/delta/chunk_recalculated/combined_backward.rs:72-84).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct dc_chunk_bwd_args {
    pub fwd: dc_chunk_args,
    pub d_y: *const f32,
    pub d_state_final: *const f32,
    pub d_q: *mut f32,
    pub d_k: *mut f32,
    pub d_v: *mut f32,
    pub d_erase: *mut f32,
    pub d_write: *mut f32,
    pub d_g: *mut f32,
    pub d_state: *mut f32,
    pub workspace: *mut c_void,
    pub workspace_bytes: u64,
}

/// `OutNorm::forward` (src/common/norm.rs:129-135).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct dc_out_norm_args {
    pub rows: i64,
    pub dv: i64,
    pub in_dtype: i32,
    pub out_dtype: i32,
    pub eps: f32,
    pub y: *const c_void,
    pub gate: *const c_void,
    pub weight: *const f32,
    pub out: *mut c_void,
}

/// The front-end after `in_proj` (src/common/qkv.rs:373-500).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct dc_qkv_prologue_args {
    pub batch: i64,
    pub seq: i64,
    pub heads: i64,
    pub dk: i64,
    pub dv: i64,
    pub n_householder: i32,
    pub conv_kernel: i32,
    pub in_dtype: i32,
    pub out_dtype: i32,
    pub flags: u32,
    pub x_stride: i64,
    pub x: *const c_void,
    pub conv_weight: *const f32,
    pub conv_bias: *const f32,
    pub window_in: *const f32,
    pub window_out: *mut f32,
    pub q: *mut c_void,
    pub k: *mut c_void,
    pub v: *mut c_void,
}

/// The gate producers (src/common/qkv.rs:333-368, src/common/gate.rs:51-59, 178-196).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct dc_gate_args {
    pub rows: i64,
    pub cols: i64,
    pub x_stride: i64,
    pub kind: i32,
    pub in_dtype: i32,
    pub group: i32,
    pub scale: f32,
    pub lo: f32,
    pub hi: f32,
    pub x: *const c_void,
    pub bias: *const f32,
    pub a_log: *const f32,
    pub out: *mut f32,
}

#[link(name = "deltacore")]
extern "C" {
    pub fn dc_chunk_fwd(args: *const dc_chunk_args, stream: dc_stream_t) -> c_int;
    pub fn dc_chunk_workspace_size(args: *const dc_chunk_args) -> u64;
    pub fn dc_chunk_kernel_choice(args: *const dc_chunk_args) -> c_int;
    pub fn dc_chunk_launches(args: *const dc_chunk_args) -> c_int;
    pub fn dc_chunk_fwd_noalloc(args: *const dc_chunk_args, stream: dc_stream_t) -> c_int;
    pub fn dc_chunk_fwd_host_scratch_size(args: *const dc_chunk_args) -> u64;
    pub fn dc_chunk_fwd_host(args: *const dc_chunk_args, scratch: *mut c_void, scratch_bytes: u64,
                             stream: dc_stream_t) -> c_int;
    pub fn dc_chunk_bwd_workspace_size(args: *const dc_chunk_bwd_args) -> u64;
    pub fn dc_chunk_bwd(args: *const dc_chunk_bwd_args, stream: dc_stream_t) -> c_int;
    pub fn dc_step(args: *const dc_step_args, stream: dc_stream_t) -> c_int;
    pub fn dc_out_norm(args: *const dc_out_norm_args, stream: dc_stream_t) -> c_int;
    pub fn dc_chunk_fwd_out_norm(chunk: *const dc_chunk_args, norm: *const dc_out_norm_args,
                                 stream: dc_stream_t) -> c_int;
    pub fn dc_chunk_fwd_out_norm_fused(chunk: *const dc_chunk_args, norm: *const dc_out_norm_args) -> c_int;
    pub fn dc_qkv_prologue(args: *const dc_qkv_prologue_args, stream: dc_stream_t) -> c_int;
    pub fn dc_gates(args: *const dc_gate_args, stream: dc_stream_t) -> c_int;
    pub fn dc_status_string(status: c_int) -> *const c_char;
    pub fn dc_last_cuda_error() -> c_int;
    pub fn dc_device_status(reset: c_int) -> c_int;
    pub fn dc_version() -> c_int;
}

/// Panic with the library's message unless `status` is `DC_OK`: the reference's error behaviour for the
/// same checks is an `assert!` panic (src/delta/path.rs:177-208).
pub fn check(status: c_int, what: &str) {
    if status != DC_OK {
        let msg = unsafe { CStr::from_ptr(dc_status_string(status)) }.to_string_lossy();
        if status == DC_ECUDA {
            let code = unsafe { dc_last_cuda_error() };
            panic!("{what}: {msg} (cudaError {code})");
        }
        panic!("{what}: {msg}");
    }
}

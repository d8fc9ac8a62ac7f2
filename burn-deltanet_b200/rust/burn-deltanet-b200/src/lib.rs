//! burn-deltanet's delta-rule core on the B200 library, for Burn's CUDA backend.
//!
//! Not compiled here: no Rust toolchain in this image, and the Burn git dependencies are not vendored.
//!
//! * [`delta_chunk_recalculated`] is the body of `DeltaChunkBackendExt::delta_chunk_recalculated`
//!   (src/delta/chunk_recalculated/chunk_recalculated.rs:105-126) for Burn's cubecl CUDA backend: the same
//!   arguments and returns, evaluated by `dc_chunk_fwd`.
//! * [`DeltaStepBackendExt`] gives the decode tick `delta_step` (src/delta/recurrent.rs:41-50), a free
//!   function on `Tensor` in the reference, a backend-extension op with the same argument list, so that
//!   every family's `step` reaches `dc_step`; `n_householder` folds DeltaProduct / GDN-2 micro-steps into
//!   the one call instead of the reference's host-built mini-sequence (src/delta_product/delta_product.rs:
//!   270-305).
//!
//! Hook point in the reference: its `#[backend_extension(Cube: cfg(...), ...)]` list
//! (chunk_recalculated.rs:86-104) generates an impl with the portable default body for every cubecl
//! runtime.  With the `b200` feature the `Cube` entry is dropped from that list and
//! `impl DeltaChunkBackendExt for Cube` is written by hand: it calls [`delta_chunk_recalculated`] when the
//! tensors live on a CUDA device with compute capability 10.0, and the portable body otherwise.  Other
//! backends (Flex, NdArray, LibTorch, Remote) and `Autodiff` (whose backward recomputes through this same
//! op, backward.rs:30-265) are unchanged.
#![allow(non_snake_case, clippy::too_many_arguments)]

pub mod handles;

use burn::tensor::ops::FloatTensor;
use deltacore_sys as sys;
use handles::{cuda_stream, dc_dtype, device_ptr, device_ptr_mut, empty, empty_bytes, shape4, CudaBackend};

/// `delta_chunk_recalculated` (chunk_recalculated.rs:115-126) on `dc_chunk_fwd`.
///
/// The reference panics on a shape or width violation (`DeltaInput::sanity`, src/delta/path.rs:177-208,
/// which runs before the op); the library returns the same checks as status codes and `sys::check` turns
/// them back into panics.  Per-channel gates (GDN-2) take the two-kernel tensor-core path, whose
/// workspace comes from Burn's own memory pool.
pub fn delta_chunk_recalculated(
    q_bshk: FloatTensor<CudaBackend>,
    k_bshk: FloatTensor<CudaBackend>,
    v_bshv: FloatTensor<CudaBackend>,
    erase_bshK: FloatTensor<CudaBackend>,
    write_bshV: FloatTensor<CudaBackend>,
    g_bshK: FloatTensor<CudaBackend>,
    state_bhkv: FloatTensor<CudaBackend>,
    has_gate: bool,
    chunk_len: usize,
    scale: f64,
) -> (FloatTensor<CudaBackend>, FloatTensor<CudaBackend>) {
    let [b, s, h, dk] = shape4(&q_bshk);
    let dv = shape4(&v_bshv)[3];
    let device = q_bshk.device.clone();
    let y = empty(&device, [b, s, h, dv], q_bshk.dtype);
    let s_out = empty(&device, [b, h, dk, dv], burn::tensor::DType::F32);
    let mut args = sys::dc_chunk_args {
        batch: b as i64,
        seq: s as i64,
        heads: h as i64,
        dk: dk as i64,
        dv: dv as i64,
        n_householder: 1,
        erase_w: shape4(&erase_bshK)[3] as i32,
        write_w: shape4(&write_bshV)[3] as i32,
        g_w: if has_gate { shape4(&g_bshK)[3] as i32 } else { 0 },
        chunk_len: chunk_len as i32,
        in_dtype: dc_dtype(&q_bshk),
        gate_dtype: dc_dtype(&erase_bshK),
        out_dtype: dc_dtype(&y),
        flags: 0,
        scale,
        q: device_ptr(&q_bshk),
        k: device_ptr(&k_bshk),
        v: device_ptr(&v_bshv),
        erase: device_ptr(&erase_bshK),
        write: device_ptr(&write_bshV),
        g: if has_gate { device_ptr(&g_bshK) } else { std::ptr::null() },
        state_in: device_ptr(&state_bhkv) as *const f32,
        y: device_ptr_mut(&y),
        state_out: device_ptr_mut(&s_out) as *mut f32,
        workspace: std::ptr::null_mut(),
        workspace_bytes: 0,
    };
    let need = unsafe { sys::dc_chunk_workspace_size(&args) };
    let ws = (need > 0).then(|| empty_bytes(&device, need as usize));
    if let Some(ws) = &ws {
        args.workspace = device_ptr_mut(ws);
        args.workspace_bytes = need;
    }
    sys::check(unsafe { sys::dc_chunk_fwd(&args, cuda_stream(&device)) }, "dc_chunk_fwd");
    // `ws` is released back to Burn's pool after the call has been enqueued on the same stream.
    (y, s_out)
}

/// The decode tick as a backend-extension op: `delta_step`'s argument list (src/delta/recurrent.rs:41-50)
/// plus `n_householder` (k, v, erase, write carry `[batch, u, heads, .]`; q and g one row per token).
pub trait DeltaStepBackendExt: burn::backend::Backend {
    fn delta_step(
        q_bhk: FloatTensor<Self>,
        k_buhk: FloatTensor<Self>,
        v_buhv: FloatTensor<Self>,
        erase_buhK: FloatTensor<Self>,
        write_buhV: FloatTensor<Self>,
        g_bhK: Option<FloatTensor<Self>>,
        state_bhkv: FloatTensor<Self>,
        scale: f64,
        n_householder: usize,
    ) -> (FloatTensor<Self>, FloatTensor<Self>);
}

impl DeltaStepBackendExt for CudaBackend {
    fn delta_step(
        q_bhk: FloatTensor<Self>,
        k_buhk: FloatTensor<Self>,
        v_buhv: FloatTensor<Self>,
        erase_buhK: FloatTensor<Self>,
        write_buhV: FloatTensor<Self>,
        g_bhK: Option<FloatTensor<Self>>,
        state_bhkv: FloatTensor<Self>,
        scale: f64,
        n_householder: usize,
    ) -> (FloatTensor<Self>, FloatTensor<Self>) {
        let dims = q_bhk.shape.dims.clone();
        let (b, h, dk) = (dims[0], dims[1], dims[2]);
        let dv = *v_buhv.shape.dims.last().unwrap();
        let device = q_bhk.device.clone();
        let y = empty(&device, [b, 1, h, dv], q_bhk.dtype);
        let s_out = empty(&device, [b, h, dk, dv], burn::tensor::DType::F32);
        let last = |t: &FloatTensor<Self>| *t.shape.dims.last().unwrap() as i32;
        let args = sys::dc_step_args {
            batch: b as i64,
            heads: h as i64,
            dk: dk as i64,
            dv: dv as i64,
            n_householder: n_householder as i32,
            erase_w: last(&erase_buhK),
            write_w: last(&write_buhV),
            g_w: g_bhK.as_ref().map_or(0, last),
            in_dtype: dc_dtype(&q_bhk),
            gate_dtype: dc_dtype(&erase_buhK),
            out_dtype: dc_dtype(&y),
            flags: 0,
            scale,
            q: device_ptr(&q_bhk),
            k: device_ptr(&k_buhk),
            v: device_ptr(&v_buhv),
            erase: device_ptr(&erase_buhK),
            write: device_ptr(&write_buhV),
            g: g_bhK.as_ref().map_or(std::ptr::null(), device_ptr),
            state_in: device_ptr(&state_bhkv) as *const f32,
            y: device_ptr_mut(&y),
            state_out: device_ptr_mut(&s_out) as *mut f32,
        };
        sys::check(unsafe { sys::dc_step(&args, cuda_stream(&device)) }, "dc_step");
        (y, s_out)
    }
}

//! The few accessors the binding needs from Burn's cubecl CUDA tensor handles, in one place.
//!
//! Not compiled here: no Rust toolchain in this image.  Written against Burn's `CubeBackend` with the
//! CUDA runtime at the reference's pinned revision (4a0d7265); a maintainer adjusts only this file if
//! those internals differ.

use burn::tensor::DType;
use burn::tensor::ops::FloatTensor;
use burn_cuda::CudaDevice;
use cubecl::cuda::CudaRuntime;
use cubecl::prelude::*;
use deltacore_sys as sys;
use std::ffi::c_void;

/// Burn's CUDA backend: cubecl's `CubeBackend` over the CUDA runtime, f32 floats, i32 ints.
pub type CudaBackend = burn::backend::cube::CubeBackend<CudaRuntime, f32, i32, u8>;

/// The four extents of a rank-4 tensor.
pub fn shape4(t: &FloatTensor<CudaBackend>) -> [usize; 4] {
    let d = &t.shape.dims;
    assert_eq!(d.len(), 4, "expected a rank-4 tensor");
    [d[0], d[1], d[2], d[3]]
}

/// The library's dtype code of a tensor: f32 or bf16, anything else is the reference's panic.
pub fn dc_dtype(t: &FloatTensor<CudaBackend>) -> i32 {
    match t.dtype {
        DType::F32 => sys::DC_F32,
        DType::BF16 => sys::DC_BF16,
        other => panic!("the B200 delta-rule core takes f32 or bf16 tensors, got {other:?}"),
    }
}

/// The tensor's device address (the `CUdeviceptr` of its binding plus its offset).  The kernels read
/// the reference's contiguous row-major layout: a strided handle is made contiguous first.
pub fn device_ptr(t: &FloatTensor<CudaBackend>) -> *const c_void {
    assert!(t.is_contiguous(), "the B200 delta-rule core reads contiguous tensors");
    let binding = t.handle.clone().binding();
    let resource = t.client.get_resource(binding);
    resource.resource().ptr as *const c_void
}

pub fn device_ptr_mut(t: &FloatTensor<CudaBackend>) -> *mut c_void {
    device_ptr(t) as *mut c_void
}

/// The CUDA stream Burn queues this device's work on (the library enqueues on the same one, so no
/// synchronisation is needed on either side).
pub fn cuda_stream(device: &CudaDevice) -> sys::dc_stream_t {
    let client = CudaRuntime::client(device);
    client.stream_handle() as sys::dc_stream_t
}

/// A new contiguous tensor of `shape` and `dtype` from Burn's memory pool.
pub fn empty(device: &CudaDevice, shape: [usize; 4], dtype: DType) -> FloatTensor<CudaBackend> {
    let client = CudaRuntime::client(device);
    let bytes = shape.iter().product::<usize>() * dtype.size();
    let handle = client.empty(bytes);
    burn::backend::cube::CubeTensor::new_contiguous(client, device.clone(), shape.into(), handle, dtype)
}

/// An untyped device buffer of `bytes` from Burn's memory pool (the two-kernel path's workspace).
pub fn empty_bytes(device: &CudaDevice, bytes: usize) -> FloatTensor<CudaBackend> {
    empty(device, [1, 1, 1, bytes.div_ceil(4)], DType::F32)
}

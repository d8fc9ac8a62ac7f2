"""ctypes binding of libdeltacore.so (the C ABI declared in include/deltacore.h).

The library is loaded from this package directory and nowhere else.  There is
no fallback: if the library is missing the import of the binding raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdeltacore.so")

# enum dc_status
DC_OK = 0
DC_EINVAL_SHAPE = 1
DC_EINVAL_WIDTH = 2
DC_EUNSUPPORTED_DTYPE = 3
DC_EINVAL_ARG = 4
DC_EUNSUPPORTED = 5
DC_ECUDA = 6
DC_EDEVICE = 7
DC_EWORKSPACE = 8
DC_ESCRATCH = 9
DC_NOALLOC_SCRATCH_BYTES = 64 << 20

# enum dc_dtype
DC_F32 = 0
DC_BF16 = 1

DC_FLAG_FORCE_SIMT = 0x1
DC_FLAG_RECURRENT = 0x2
DC_FLAG_FORCE_SPLIT = 0x4
DC_FLAG_TEST_STALL = 0x100

EXPORTS = (
    "dc_chunk_fwd", "dc_step", "dc_status_string", "dc_last_cuda_error", "dc_device_status",
    "dc_chunk_kernel_choice", "dc_chunk_launches", "dc_version", "dc_chunk_workspace_size",
    "dc_chunk_fwd_noalloc",
    "dc_chunk_fwd_host_scratch_size",
    "dc_chunk_fwd_host",
    "dc_chunk_bwd_workspace_size",
    "dc_chunk_bwd",
    "dc_out_norm",
    "dc_chunk_fwd_out_norm",
    "dc_chunk_fwd_out_norm_fused",
    "dc_qkv_prologue",
    "dc_gates",
)


class ChunkArgs(ctypes.Structure):
    """struct dc_chunk_args."""
    _fields_ = [
        ("batch", ctypes.c_int64), ("seq", ctypes.c_int64), ("heads", ctypes.c_int64),
        ("dk", ctypes.c_int64), ("dv", ctypes.c_int64),
        ("n_householder", ctypes.c_int32),
        ("erase_w", ctypes.c_int32), ("write_w", ctypes.c_int32), ("g_w", ctypes.c_int32),
        ("chunk_len", ctypes.c_int32),
        ("in_dtype", ctypes.c_int32), ("gate_dtype", ctypes.c_int32), ("out_dtype", ctypes.c_int32),
        ("flags", ctypes.c_uint32),
        ("scale", ctypes.c_double),
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("erase", ctypes.c_void_p), ("write", ctypes.c_void_p), ("g", ctypes.c_void_p),
        ("state_in", ctypes.c_void_p), ("y", ctypes.c_void_p), ("state_out", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_uint64),
    ]


class ChunkBwdArgs(ctypes.Structure):
    """struct dc_chunk_bwd_args."""
    _fields_ = [
        ("fwd", ChunkArgs),
        ("d_y", ctypes.c_void_p), ("d_state_final", ctypes.c_void_p),
        ("d_q", ctypes.c_void_p), ("d_k", ctypes.c_void_p), ("d_v", ctypes.c_void_p),
        ("d_erase", ctypes.c_void_p), ("d_write", ctypes.c_void_p), ("d_g", ctypes.c_void_p),
        ("d_state", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_uint64),
    ]


class StepArgs(ctypes.Structure):
    """struct dc_step_args."""
    _fields_ = [
        ("batch", ctypes.c_int64), ("heads", ctypes.c_int64), ("dk", ctypes.c_int64), ("dv", ctypes.c_int64),
        ("n_householder", ctypes.c_int32),
        ("erase_w", ctypes.c_int32), ("write_w", ctypes.c_int32), ("g_w", ctypes.c_int32),
        ("in_dtype", ctypes.c_int32), ("gate_dtype", ctypes.c_int32), ("out_dtype", ctypes.c_int32),
        ("flags", ctypes.c_uint32),
        ("scale", ctypes.c_double),
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("erase", ctypes.c_void_p), ("write", ctypes.c_void_p), ("g", ctypes.c_void_p),
        ("state_in", ctypes.c_void_p), ("y", ctypes.c_void_p), ("state_out", ctypes.c_void_p),
    ]


class OutNormArgs(ctypes.Structure):
    """struct dc_out_norm_args."""
    _fields_ = [
        ("rows", ctypes.c_int64), ("dv", ctypes.c_int64),
        ("in_dtype", ctypes.c_int32), ("out_dtype", ctypes.c_int32),
        ("eps", ctypes.c_float),
        ("y", ctypes.c_void_p), ("gate", ctypes.c_void_p), ("weight", ctypes.c_void_p), ("out", ctypes.c_void_p),
    ]


DC_PROLOGUE_CONV_SILU = 0x1
DC_PROLOGUE_QK_SILU = 0x2
DC_PROLOGUE_L2 = 0x4


class PrologueArgs(ctypes.Structure):
    """struct dc_qkv_prologue_args."""
    _fields_ = [
        ("batch", ctypes.c_int64), ("seq", ctypes.c_int64), ("heads", ctypes.c_int64),
        ("dk", ctypes.c_int64), ("dv", ctypes.c_int64),
        ("n_householder", ctypes.c_int32), ("conv_kernel", ctypes.c_int32),
        ("in_dtype", ctypes.c_int32), ("out_dtype", ctypes.c_int32),
        ("flags", ctypes.c_uint32),
        ("x_stride", ctypes.c_int64),
        ("x", ctypes.c_void_p), ("conv_weight", ctypes.c_void_p), ("conv_bias", ctypes.c_void_p),
        ("window_in", ctypes.c_void_p), ("window_out", ctypes.c_void_p),
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
    ]


DC_GATE_WRITE = 0
DC_GATE_HEAD_DECAY = 1
DC_GATE_CHANNEL_DECAY = 2


class GateArgs(ctypes.Structure):
    """struct dc_gate_args."""
    _fields_ = [
        ("rows", ctypes.c_int64), ("cols", ctypes.c_int64), ("x_stride", ctypes.c_int64),
        ("kind", ctypes.c_int32), ("in_dtype", ctypes.c_int32), ("group", ctypes.c_int32),
        ("scale", ctypes.c_float), ("lo", ctypes.c_float), ("hi", ctypes.c_float),
        ("x", ctypes.c_void_p), ("bias", ctypes.c_void_p), ("a_log", ctypes.c_void_p), ("out", ctypes.c_void_p),
    ]


_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library.  Raises OSError if libdeltacore.so was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is missing: build it with `python burn-deltanet_b200/build.py` "
                          "(the delta-rule core has no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        L.dc_chunk_fwd.argtypes = [ctypes.POINTER(ChunkArgs), ctypes.c_void_p]
        L.dc_chunk_fwd.restype = ctypes.c_int
        L.dc_step.argtypes = [ctypes.POINTER(StepArgs), ctypes.c_void_p]
        L.dc_step.restype = ctypes.c_int
        L.dc_status_string.argtypes = [ctypes.c_int]
        L.dc_status_string.restype = ctypes.c_char_p
        L.dc_last_cuda_error.argtypes = []
        L.dc_last_cuda_error.restype = ctypes.c_int
        L.dc_device_status.argtypes = [ctypes.c_int]
        L.dc_device_status.restype = ctypes.c_int
        L.dc_chunk_kernel_choice.argtypes = [ctypes.POINTER(ChunkArgs)]
        L.dc_chunk_kernel_choice.restype = ctypes.c_int
        L.dc_chunk_launches.argtypes = [ctypes.POINTER(ChunkArgs)]
        L.dc_chunk_launches.restype = ctypes.c_int
        L.dc_version.argtypes = []
        L.dc_version.restype = ctypes.c_int
        L.dc_chunk_workspace_size.argtypes = [ctypes.POINTER(ChunkArgs)]
        L.dc_chunk_workspace_size.restype = ctypes.c_uint64
        L.dc_chunk_fwd_noalloc.argtypes = [ctypes.POINTER(ChunkArgs), ctypes.c_void_p]
        L.dc_chunk_fwd_noalloc.restype = ctypes.c_int
        L.dc_chunk_fwd_host_scratch_size.argtypes = [ctypes.POINTER(ChunkArgs)]
        L.dc_chunk_fwd_host_scratch_size.restype = ctypes.c_uint64
        L.dc_chunk_fwd_host.argtypes = [ctypes.POINTER(ChunkArgs), ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]
        L.dc_chunk_fwd_host.restype = ctypes.c_int
        L.dc_chunk_bwd_workspace_size.argtypes = [ctypes.POINTER(ChunkBwdArgs)]
        L.dc_chunk_bwd_workspace_size.restype = ctypes.c_uint64
        L.dc_chunk_bwd.argtypes = [ctypes.POINTER(ChunkBwdArgs), ctypes.c_void_p]
        L.dc_chunk_bwd.restype = ctypes.c_int
        L.dc_out_norm.argtypes = [ctypes.POINTER(OutNormArgs), ctypes.c_void_p]
        L.dc_out_norm.restype = ctypes.c_int
        L.dc_chunk_fwd_out_norm.argtypes = [ctypes.POINTER(ChunkArgs), ctypes.POINTER(OutNormArgs), ctypes.c_void_p]
        L.dc_chunk_fwd_out_norm.restype = ctypes.c_int
        L.dc_chunk_fwd_out_norm_fused.argtypes = [ctypes.POINTER(ChunkArgs), ctypes.POINTER(OutNormArgs)]
        L.dc_chunk_fwd_out_norm_fused.restype = ctypes.c_int
        L.dc_qkv_prologue.argtypes = [ctypes.POINTER(PrologueArgs), ctypes.c_void_p]
        L.dc_qkv_prologue.restype = ctypes.c_int
        L.dc_gates.argtypes = [ctypes.POINTER(GateArgs), ctypes.c_void_p]
        L.dc_gates.restype = ctypes.c_int
        _lib = L
    return _lib


def status_string(status: int) -> str:
    return lib().dc_status_string(status).decode()

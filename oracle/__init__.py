"""CPU oracle for burn-deltanet's delta-rule core.

TEST INFRASTRUCTURE ONLY.  This package is the parity checker for the CUDA
kernels and the timed CPU baseline of ``bench.py``.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and its
``--impl reference`` arm) may import it; the product package never does.

It wraps ``liboracle.so`` (``oracle_core.c``, built by ``oracle/Makefile``):

* ``recurrent``  — src/delta/recurrent.rs:41-142 (the definition);
* ``chunk``      — src/delta/chunk.rs:41-221, with decay.rs:82-143 and
  tri.rs:72-136 (the reference's chunkwise WY forward);
* ``fold`` / ``unfold`` — the DeltaProduct / GDN-2 micro-step fold of
  src/delta_product/delta_product.rs:178-228 (q on the last micro-step, the
  forget gate on the first, the output of the last micro-step kept);
* ``recurrent_backward`` (``oracle/backward.py``, numpy) — the gradients of
  the custom backward (src/delta/chunk_recalculated/combined_backward.rs:
  72-190) as the derivative of the recurrence, float64;
* ``out_norm`` (``oracle/out_norm.py``, numpy) — the per-head output
  normalisation OutNorm (src/common/norm.rs:106-144);
* ``qkv_prologue`` (``oracle/prologue.py``, numpy) — the front-end after the
  input projection: short convolution, activations, q/k L2 norm
  (src/common/conv.rs, src/common/qkv.rs:373-500), and its gate producers
  ``write_gate`` / ``head_log_decay`` / ``channel_log_decay``
  (qkv.rs:333-368, src/common/gate.rs:51-59, 178-196).

Arrays use the reference's layouts: per-token ``[batch, seq, heads, width]``,
state ``[batch, heads, dk, dv]``.

Parity pin: tests/test_oracle_golden.py checks the float64 build against the
reference's own float64 golden vectors (src/delta/tests/reference.rs).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")


class _Dims(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_long), ("seq", ctypes.c_long), ("heads", ctypes.c_long),
        ("dk", ctypes.c_long), ("dv", ctypes.c_long),
        ("erase_w", ctypes.c_long), ("write_w", ctypes.c_long), ("g_w", ctypes.c_long),
        ("scale", ctypes.c_double), ("threads", ctypes.c_int),
    ]


def build() -> str:
    """Compile liboracle.so with oracle/Makefile; returns its path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        for name, real in (("f64", ctypes.c_double), ("f32", ctypes.c_float)):
            p = ctypes.POINTER(real)
            fn = getattr(_lib, f"orc_recurrent_{name}")
            fn.argtypes = [ctypes.POINTER(_Dims)] + [p] * 9
            fn.restype = None
            fn = getattr(_lib, f"orc_chunk_{name}")
            fn.argtypes = [ctypes.POINTER(_Dims), ctypes.c_long] + [p] * 9
            fn.restype = None
        _lib.orc_unit_lower_inverse_f64.argtypes = [
            ctypes.c_long, ctypes.c_long, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]
        _lib.orc_unit_lower_inverse_f64.restype = None
    return _lib


def _ptr(a, real):
    if a is None:
        return ctypes.cast(None, ctypes.POINTER(real))
    return a.ctypes.data_as(ctypes.POINTER(real))


def _prep(q, k, v, erase, write, g, state, scale, dtype):
    arrs = [np.ascontiguousarray(x, dtype=dtype) if x is not None else None
            for x in (q, k, v, erase, write, g, state)]
    q, k, v, erase, write, g, state = arrs
    b, s, h, dk = q.shape
    dv = v.shape[3]
    assert k.shape == (b, s, h, dk) and v.shape == (b, s, h, dv)
    assert state.shape == (b, h, dk, dv)
    assert erase.shape[:3] == (b, s, h) and erase.shape[3] in (1, dk)
    assert write.shape[:3] == (b, s, h) and write.shape[3] in (1, dv)
    if g is not None:
        assert g.shape[:3] == (b, s, h) and g.shape[3] in (1, dk)
    dims = _Dims(b, s, h, dk, dv, erase.shape[3], write.shape[3], 0 if g is None else g.shape[3],
                 float(1.0 / np.sqrt(dk) if scale is None else scale), 0)
    return arrs, dims


def _run(kind, q, k, v, erase, write, g, state, scale, chunk_len, dtype, threads):
    real = ctypes.c_double if dtype == np.float64 else ctypes.c_float
    name = "f64" if dtype == np.float64 else "f32"
    (q, k, v, erase, write, g, state), dims = _prep(q, k, v, erase, write, g, state, scale, dtype)
    dims.threads = int(threads or 0)
    b, s, h, _ = q.shape
    y = np.empty((b, s, h, v.shape[3]), dtype=dtype)
    s_out = np.empty_like(state)
    args = [_ptr(x, real) for x in (q, k, v, erase, write, g, state, y, s_out)]
    if kind == "recurrent":
        getattr(lib(), f"orc_recurrent_{name}")(ctypes.byref(dims), *args)
    else:
        assert chunk_len >= 1
        getattr(lib(), f"orc_chunk_{name}")(ctypes.byref(dims), int(chunk_len), *args)
    return y, s_out


def recurrent(q, k, v, erase, write, g, state, scale=None, dtype=np.float64, threads=0):
    """DeltaPath::Recurrent (src/delta/recurrent.rs:107-142). Returns (y, final_state)."""
    return _run("recurrent", q, k, v, erase, write, g, state, scale, 1, dtype, threads)


def chunk(q, k, v, erase, write, g, state, chunk_len=64, scale=None, dtype=np.float64, threads=0):
    """DeltaPath::Chunk{chunk_len, Blocked} (src/delta/chunk.rs:41-221). Returns (y, final_state)."""
    return _run("chunk", q, k, v, erase, write, g, state, scale, chunk_len, dtype, threads)


def step(q, k, v, erase, write, g, state, scale=None, dtype=np.float64):
    """delta_step (src/delta/recurrent.rs:41-99) on [batch, heads, width] inputs."""
    add = lambda x: None if x is None else np.asarray(x)[:, None]
    y, s = recurrent(add(q), add(k), add(v), add(erase), add(write), add(g), state, scale, dtype)
    return y[:, 0], s


def unit_lower_inverse(n_strict):
    """TriSolve::Blocked (src/delta/tri.rs:72-114) on [..., size, size]."""
    n = np.ascontiguousarray(n_strict, dtype=np.float64)
    size = n.shape[-1]
    flat = n.reshape(-1, size, size)
    out = np.empty_like(flat)
    lib().orc_unit_lower_inverse_f64(flat.shape[0], size, _ptr(flat, ctypes.c_double),
                                     _ptr(out, ctypes.c_double))
    return out.reshape(n.shape)


# ---------------------------------------------------------------------------
# The micro-step fold (src/delta_product/delta_product.rs:178-228, :270-305;
# src/gated_deltanet_2/gated_deltanet_2.rs:225-271).
# ---------------------------------------------------------------------------
def fold(q_bthk, g_bthK, u):
    """Spread per-token q and g over u micro-steps, as the families do before
    calling the core: q sits on the last micro-step and g on the first, zeros
    elsewhere.  Returns (q_folded [b, t*u, h, dk], g_folded or None)."""
    q = np.asarray(q_bthk)
    b, t, h, dk = q.shape
    if u == 1:
        return q, g_bthK
    qf = np.zeros((b, t, u, h, dk), dtype=q.dtype)
    qf[:, :, u - 1] = q
    gf = None
    if g_bthK is not None:
        g = np.asarray(g_bthK)
        gf = np.zeros((b, t, u, h, g.shape[3]), dtype=g.dtype)
        gf[:, :, 0] = g
        gf = gf.reshape(b, t * u, h, g.shape[3])
    return qf.reshape(b, t * u, h, dk), gf


def unfold(y_bTv, u):
    """Keep each token's last micro-step output: [b, t*u, h, dv] -> [b, t, h, dv]."""
    y = np.asarray(y_bTv)
    b, tu, h, dv = y.shape
    return y.reshape(b, tu // u, u, h, dv)[:, :, u - 1]


def householder(kind, q, k, v, erase, write, g, state, u, chunk_len=64, scale=None,
                 dtype=np.float64, threads=0):
    """Run the core on a micro-step-folded sequence.  k, v, erase, write carry
    t*u rows; q and g carry t rows.  Returns (y [b, t, h, dv], final_state)."""
    qf, gf = fold(q, g, u)
    if scale is None:
        scale = 1.0 / np.sqrt(np.asarray(q).shape[3])
    if kind == "recurrent":
        y, s = recurrent(qf, k, v, erase, write, gf, state, scale, dtype, threads)
    else:
        y, s = chunk(qf, k, v, erase, write, gf, state, chunk_len, scale, dtype, threads)
    return unfold(y, u), s


from .backward import recurrent_backward  # noqa: E402  (numpy only)
from .out_norm import out_norm  # noqa: E402  (numpy only)
from .prologue import channel_log_decay, head_log_decay, qkv_prologue, softplus, write_gate  # noqa: E402

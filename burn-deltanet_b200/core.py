"""Host-side mirror of burn-deltanet's delta-rule core interface.

Same names, argument meaning and error behaviour as the reference's
``src/delta`` public surface (src/delta/mod.rs:132-137), on CUDA tensors:

* :class:`DeltaPath`  — src/delta/path.rs:21-99
* :class:`TriSolve`   — src/delta/tri.rs:53-64
* :class:`DeltaInput` — src/delta/path.rs:120-231 (``dims``, ``resolved_scale``,
  ``has_channel_decay``, ``sanity``, ``run``)
* :func:`beta_gates`  — src/delta/path.rs:147-150
* :func:`delta_step`  — src/delta/recurrent.rs:41-99
* :func:`delta_chunk_recalculated` — the backend-extension op
  ``DeltaChunkBackendExt::delta_chunk_recalculated``
  (src/delta/chunk_recalculated/chunk_recalculated.rs:115-126)

Every evaluation goes through the C ABI in libdeltacore.so; the reference's
``assert!`` panics become :class:`DeltaCoreError` (``DeltaShapeError`` for the
shape and width checks).  There is no CPU path: CPU tensors are rejected.

One extension over the reference: ``n_householder`` (DeltaProduct's ``u``)
folds the micro-steps inside the kernel instead of building the zero-padded
sequence on the host (src/delta_product/delta_product.rs:178-228).  With
``n_householder == 1`` (the default) the arguments are the reference's.
"""
from __future__ import annotations

import enum
import math
import os
from dataclasses import dataclass
from typing import Optional, Tuple

import torch

from . import _abi


class DeltaCoreError(RuntimeError):
    """A status other than DC_OK from the C ABI."""

    def __init__(self, status: int, what: str = ""):
        self.status = status
        msg = _abi.status_string(status)
        if status == _abi.DC_ECUDA:
            msg += f" (cudaError {_abi.lib().dc_last_cuda_error()})"
        super().__init__(f"{what}: {msg}" if what else msg)


class DeltaShapeError(DeltaCoreError, ValueError):
    """The shape / width checks of DeltaInput::sanity (src/delta/path.rs:177-208)."""


class DeltaNonFiniteError(DeltaCoreError, ValueError):
    """A NaN or Inf found by the opt-in guard (see :func:`set_sanity_checks`)."""


# The reference compiles its NaN / Inf guard in only under its `check-nan` / `check-inf` features
# (burn-stack's `sanity`, called at src/delta/path.rs:198-207 and src/delta/recurrent.rs:96-97).  Here the
# same guard is off by default and switched on per process, by set_sanity_checks() or the environment
# variables DELTACORE_CHECK_NAN=1 / DELTACORE_CHECK_INF=1.  Each check is one device reduction over the
# tensor and a host read of its result, so it synchronises the stream: a debugging aid, as in the reference.
_SANITY = {"nan": os.environ.get("DELTACORE_CHECK_NAN", "0") not in ("", "0"),
           "inf": os.environ.get("DELTACORE_CHECK_INF", "0") not in ("", "0")}


def set_sanity_checks(nan: bool = True, inf: bool = True) -> None:
    """Switch the NaN / Inf guard of ``DeltaInput.sanity`` and ``delta_step`` on or off."""
    _SANITY["nan"], _SANITY["inf"] = bool(nan), bool(inf)


def san(t: Optional[torch.Tensor], what: str) -> None:
    """Raise :class:`DeltaNonFiniteError` if ``t`` holds a NaN (check-nan) or an Inf (check-inf)."""
    if t is None or not (_SANITY["nan"] or _SANITY["inf"]):
        return
    if _SANITY["nan"] and bool(torch.isnan(t).any()):
        raise DeltaNonFiniteError(_abi.DC_EINVAL_ARG, f"{what} holds NaN")
    if _SANITY["inf"] and bool(torch.isinf(t).any()):
        raise DeltaNonFiniteError(_abi.DC_EINVAL_ARG, f"{what} holds Inf")


def _raise(status: int, what: str) -> None:
    if status == _abi.DC_OK:
        return
    if status in (_abi.DC_EINVAL_SHAPE, _abi.DC_EINVAL_WIDTH):
        raise DeltaShapeError(status, what)
    raise DeltaCoreError(status, what)


class TriSolve(enum.Enum):
    """How (I - N)^-1 is evaluated (src/delta/tri.rs:53-64).  The kernels always
    substitute; both variants compute the same T and are accepted for parity."""
    Blocked = "blocked"
    Neumann = "neumann"


@dataclass(frozen=True)
class DeltaPath:
    """Which evaluation of the delta rule runs (src/delta/path.rs:21-99).

    ``kind`` is ``"recurrent"``, ``"chunk"`` or ``"chunk_recalculated"`` (the
    default).  ``Recurrent`` runs the fused step kernel token by token;
    both chunk kinds run the chunkwise prefill kernel (their forwards are
    identical in the reference, path.rs:39-45)."""
    kind: str = "chunk_recalculated"
    chunk_len: Optional[int] = None
    solve: TriSolve = TriSolve.Blocked

    DEFAULT_CHUNK_LEN = 64

    @classmethod
    def Recurrent(cls) -> "DeltaPath":
        return cls("recurrent", None)

    @classmethod
    def Chunk(cls, chunk_len: Optional[int] = None, solve: TriSolve = TriSolve.Blocked) -> "DeltaPath":
        return cls("chunk", chunk_len, solve)

    @classmethod
    def ChunkRecalculated(cls, chunk_len: Optional[int] = None) -> "DeltaPath":
        return cls("chunk_recalculated", chunk_len)

    @classmethod
    def default(cls) -> "DeltaPath":
        return cls.ChunkRecalculated(None)

    @classmethod
    def chunk(cls) -> "DeltaPath":
        return cls.default()

    @classmethod
    def with_chunk_len(cls, chunk_len: int) -> "DeltaPath":
        """``DeltaPath::chunk_len`` (path.rs:74-78)."""
        return cls.ChunkRecalculated(chunk_len)

    @classmethod
    def chunk_len_on_tape(cls, chunk_len: int) -> "DeltaPath":
        return cls.Chunk(chunk_len)

    def resolved_chunk_len(self) -> int:
        if self.kind == "recurrent":
            return 1
        return self.chunk_len if self.chunk_len is not None else self.DEFAULT_CHUNK_LEN


def _dtype_code(t: torch.Tensor, what: str) -> int:
    if t.dtype == torch.float32:
        return _abi.DC_F32
    if t.dtype == torch.bfloat16:
        return _abi.DC_BF16
    raise DeltaCoreError(_abi.DC_EUNSUPPORTED_DTYPE, f"{what} has dtype {t.dtype}")


def _check_tensor(t: torch.Tensor, what: str) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{what} must be a torch.Tensor")
    if not t.is_cuda:
        raise DeltaCoreError(_abi.DC_EDEVICE, f"{what} is on {t.device}: the delta-rule core runs on CUDA only")
    if not t.is_contiguous():
        raise DeltaCoreError(_abi.DC_EINVAL_ARG, f"{what} must be contiguous")


def _same_dtype(ts, what: str) -> int:
    codes = {_dtype_code(t, what) for t in ts if t is not None}
    if len(codes) != 1:
        raise DeltaCoreError(_abi.DC_EUNSUPPORTED_DTYPE, f"{what} must share one dtype")
    return codes.pop()


def beta_gates(beta: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """The (erase, write) pair a per-head beta stands for (src/delta/path.rs:147-150)."""
    gate = beta.unsqueeze(-1)
    return gate, gate


def _chunk_args(q_bshk, k_bshk, v_bshv, erase_bshK, write_bshV, g_bshK, state_bhkv, has_gate, chunk_len, scale,
                n_householder, out_dtype, force_simt, recurrent, force_split, y_out, state_out, check, alloc):
    """dc_chunk_args for one call, after the reference's shape / width asserts
    (path.rs:177-208); `check` validates each tensor's placement, `alloc`
    makes the outputs not given."""
    ts = dict(q=q_bshk, k=k_bshk, v=v_bshv, erase=erase_bshK, write=write_bshV, state=state_bhkv)
    if has_gate:
        ts["g"] = g_bshK
    for name, t in ts.items():
        check(t, name)
    if q_bshk.dim() != 4 or v_bshv.dim() != 4 or state_bhkv.dim() != 4:
        raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, "q, v and state must be rank 4")
    b, s, h, dk = q_bshk.shape
    dv = v_bshv.shape[3]
    u = int(n_householder)
    want = {
        "k": (b, s * u, h, dk), "v": (b, s * u, h, dv), "state": (b, h, dk, dv),
    }
    for name, shape in want.items():
        if tuple(ts[name].shape) != shape:
            raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, f"{name} has shape {tuple(ts[name].shape)}, want {shape}")
    for name, rows, full in (("erase", s * u, dk), ("write", s * u, dv)) + ((("g", s, dk),) if has_gate else ()):
        t = ts[name]
        if t.dim() != 4 or tuple(t.shape[:3]) != (b, rows, h):
            raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, f"{name} has shape {tuple(t.shape)}")
        if t.shape[3] not in (1, full):
            raise DeltaShapeError(_abi.DC_EINVAL_WIDTH, f"{name}: last axis must be 1 or {full}, got {t.shape[3]}")
    if state_bhkv.dtype != torch.float32:
        raise DeltaCoreError(_abi.DC_EUNSUPPORTED_DTYPE, "the state is float32")
    in_dt = _same_dtype((q_bshk, k_bshk, v_bshv), "q, k, v")
    gate_dt = _same_dtype((erase_bshK, write_bshV, g_bshK if has_gate else None), "erase, write, g")
    out_torch = out_dtype or q_bshk.dtype
    y = y_out if y_out is not None else alloc((b, s, h, dv), out_torch)
    s_out = state_out if state_out is not None else alloc(tuple(state_bhkv.shape), torch.float32)
    check(y, "y_out")
    check(s_out, "state_out")
    a = _abi.ChunkArgs()
    a.batch, a.seq, a.heads, a.dk, a.dv = b, s, h, dk, dv
    a.n_householder = u
    a.erase_w, a.write_w = erase_bshK.shape[3], write_bshV.shape[3]
    a.g_w = g_bshK.shape[3] if has_gate else 0
    a.chunk_len = int(chunk_len)
    a.in_dtype, a.gate_dtype, a.out_dtype = in_dt, gate_dt, _dtype_code(y, "y")
    a.flags = ((_abi.DC_FLAG_FORCE_SIMT if force_simt else 0) | (_abi.DC_FLAG_RECURRENT if recurrent else 0)
               | (_abi.DC_FLAG_FORCE_SPLIT if force_split else 0))
    a.scale = float(scale)
    a.q, a.k, a.v = q_bshk.data_ptr(), k_bshk.data_ptr(), v_bshv.data_ptr()
    a.erase, a.write = erase_bshK.data_ptr(), write_bshV.data_ptr()
    a.g = g_bshK.data_ptr() if has_gate else None
    a.state_in, a.y, a.state_out = state_bhkv.data_ptr(), y.data_ptr(), s_out.data_ptr()
    return a, y, s_out


def delta_chunk_recalculated(q_bshk, k_bshk, v_bshv, erase_bshK, write_bshV, g_bshK, state_bhkv,
                             has_gate: bool, chunk_len: int, scale: float, *, n_householder: int = 1,
                             out_dtype: Optional[torch.dtype] = None, force_simt: bool = False,
                             recurrent: bool = False, force_split: bool = False,
                             workspace: Optional[torch.Tensor] = None,
                             y_out: Optional[torch.Tensor] = None, state_out: Optional[torch.Tensor] = None):
    """The backend-extension op (chunk_recalculated.rs:115-126) on CUDA tensors.

    Shapes: q [b, s, h, dk]; k [b, s*u, h, dk]; v [b, s*u, h, dv];
    erase [b, s*u, h, 1|dk]; write [b, s*u, h, 1|dv]; g [b, s, h, 1|dk]
    (ignored unless ``has_gate``); state [b, h, dk, dv] float32.
    Returns ``(y [b, s, h, dv], final_state [b, h, dk, dv])`` as new tensors
    unless ``y_out`` / ``state_out`` are given (``state_out`` may be ``state_bhkv``).
    ``recurrent=True`` evaluates DeltaPath::Recurrent: the fused decode tick walks
    the sequence token by token (one launch per token).
    Per-channel gates (GDN-2) run on the tensor cores through a device workspace
    of ``dc_chunk_workspace_size`` bytes: pass ``workspace`` (a uint8 CUDA tensor)
    to reuse one, otherwise this layer allocates it for the call.
    ``force_split=True`` takes that two-kernel path for per-head gates too.
    """
    a, y, s_out = _chunk_args(q_bshk, k_bshk, v_bshv, erase_bshK, write_bshV, g_bshK, state_bhkv, has_gate,
                              chunk_len, scale, n_householder, out_dtype, force_simt, recurrent, force_split,
                              y_out, state_out, _check_tensor,
                              lambda shape, dt: torch.empty(shape, device=q_bshk.device, dtype=dt))
    need = int(_abi.lib().dc_chunk_workspace_size(a))
    if need > 0:
        if workspace is None:
            workspace = torch.empty(need, dtype=torch.uint8, device=q_bshk.device)
        _check_tensor(workspace, "workspace")
        a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    with torch.cuda.device(q_bshk.device):
        stream = torch.cuda.current_stream(q_bshk.device).cuda_stream
        _raise(_abi.lib().dc_chunk_fwd(a, stream), "dc_chunk_fwd")
    return y, s_out


def _norm_args(a, y, norm_weight, norm_gate, norm_eps):
    """dc_out_norm_args for the norm that follows the prefill call `a` (rows of y [b, s, h, dv])."""
    _check_tensor(norm_weight, "norm_weight")
    if norm_weight.dtype != torch.float32 or tuple(norm_weight.shape) != (a.dv,):
        raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, f"norm_weight must be float32 [{a.dv}]")
    n = _abi.OutNormArgs()
    n.rows, n.dv = a.batch * a.seq * a.heads, a.dv
    n.in_dtype, n.out_dtype, n.eps = a.out_dtype, a.out_dtype, float(norm_eps)
    n.weight = norm_weight.data_ptr()
    if norm_gate is not None:
        _check_tensor(norm_gate, "norm_gate")
        if norm_gate.shape != y.shape or _dtype_code(norm_gate, "norm_gate") != a.out_dtype:
            raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, "norm_gate must be shaped like y, in y's dtype")
        n.gate = norm_gate.data_ptr()
    return n


def delta_chunk_recalculated_out_norm(q_bshk, k_bshk, v_bshv, erase_bshK, write_bshV, g_bshK, state_bhkv,
                                      has_gate: bool, chunk_len: int, scale: float, norm_weight: torch.Tensor,
                                      norm_gate: Optional[torch.Tensor] = None, norm_eps: float = 1e-5, *,
                                      n_householder: int = 1, out_dtype: Optional[torch.dtype] = None,
                                      workspace: Optional[torch.Tensor] = None,
                                      y_out: Optional[torch.Tensor] = None,
                                      state_out: Optional[torch.Tensor] = None):
    """The prefill followed by the block's output norm (``dc_chunk_fwd_out_norm``): what a layer's
    forward does with the core's read-out before out_proj (src/common/norm.rs:129-135 on the y of
    chunk_recalculated.rs:115-126).

    Arguments as :func:`delta_chunk_recalculated`, plus the norm's float32 ``norm_weight`` [dv], its
    gate (``None``: OutNorm::Plain; else shaped like y, in y's dtype) and eps.  Returns
    ``(normalised y, final_state)``.  A plain norm on the fused tensor-core path is applied inside the
    kernel's read-out (:func:`chunk_out_norm_is_fused` says which); otherwise the call is the prefill
    followed by :func:`out_norm` in place on y.
    """
    a, y, s_out = _chunk_args(q_bshk, k_bshk, v_bshv, erase_bshK, write_bshV, g_bshK, state_bhkv, has_gate,
                              chunk_len, scale, n_householder, out_dtype, False, False, False, y_out, state_out,
                              _check_tensor, lambda shape, dt: torch.empty(shape, device=q_bshk.device, dtype=dt))
    n = _norm_args(a, y, norm_weight, norm_gate, norm_eps)
    need = int(_abi.lib().dc_chunk_workspace_size(a))
    if need > 0:
        if workspace is None:
            workspace = torch.empty(need, dtype=torch.uint8, device=q_bshk.device)
        _check_tensor(workspace, "workspace")
        a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    with torch.cuda.device(q_bshk.device):
        stream = torch.cuda.current_stream(q_bshk.device).cuda_stream
        _raise(_abi.lib().dc_chunk_fwd_out_norm(a, n, stream), "dc_chunk_fwd_out_norm")
    return y, s_out


def chunk_out_norm_is_fused(q_bshk, k_bshk, v_bshv, erase_bshK, write_bshV, g_bshK, state_bhkv,
                            has_gate: bool, chunk_len: int, norm_weight: torch.Tensor,
                            norm_gate: Optional[torch.Tensor] = None, *, n_householder: int = 1,
                            out_dtype: Optional[torch.dtype] = None) -> bool:
    """Whether :func:`delta_chunk_recalculated_out_norm` applies the norm inside the prefill kernel for
    these arguments (``dc_chunk_fwd_out_norm_fused``; host logic, nothing runs)."""
    a, y, _ = _chunk_args(q_bshk, k_bshk, v_bshv, erase_bshK, write_bshV, g_bshK, state_bhkv, has_gate,
                          chunk_len, 1.0, n_householder, out_dtype, False, False, False, None, None,
                          lambda t, what: None, lambda shape, dt: torch.empty(shape, device="meta", dtype=dt))
    a.y, a.state_out = 256, 512  # aligned placeholders, distinct from the inputs: the query reads no pointer
    n = _norm_args(a, y, norm_weight, norm_gate, 1e-5)
    r = int(_abi.lib().dc_chunk_fwd_out_norm_fused(a, n))
    if r < 0:
        _raise(-r, "dc_chunk_fwd_out_norm_fused")
    return r == 1


def delta_chunk_recalculated_backward(d_y_bshv, d_final_state_bhkv, q_bshk, k_bshk, v_bshv, erase_bshK,
                                      write_bshV, g_bshK, state_bhkv, has_gate: bool, chunk_len: int,
                                      scale: float, *, n_householder: int = 1,
                                      workspace: Optional[torch.Tensor] = None, recurrent: bool = False):
    """The backward of :func:`delta_chunk_recalculated` (``dc_chunk_bwd``): the
    reference's ``combined_backward`` (src/delta/chunk_recalculated/
    combined_backward.rs:72-84) on CUDA tensors.

    Returns ``(d_q, d_k, d_v, d_erase, d_write, d_g, d_state)`` (float32, each
    shaped like its input; ``d_g`` is ``None`` unless ``has_gate``): the
    derivatives of ``<y, d_y> + <final_state, d_final_state>`` through the
    forward call with the given inputs.  ``d_final_state_bhkv`` may be
    ``None`` (zero).  dk, dv <= 128.  A log-decay per head (or none) takes the
    chunked backward; per-channel log-decays, or ``recurrent=True``, the
    token-by-token one.
    """
    # (the forward's y / final state are not used: one-element stand-ins)
    a, _, _ = _chunk_args(q_bshk, k_bshk, v_bshv, erase_bshK, write_bshV, g_bshK, state_bhkv, has_gate,
                          chunk_len, scale, n_householder, torch.float32, False, recurrent, False, None, None,
                          _check_tensor, lambda shape, dt: torch.empty(1, device=q_bshk.device, dtype=dt))
    _check_tensor(d_y_bshv, "d_y")
    if d_y_bshv.dtype != torch.float32 or tuple(d_y_bshv.shape) != (a.batch, a.seq, a.heads, a.dv):
        raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, f"d_y must be float32 [{a.batch}, {a.seq}, {a.heads}, {a.dv}]")
    if d_final_state_bhkv is not None:
        _check_tensor(d_final_state_bhkv, "d_final_state")
        if d_final_state_bhkv.dtype != torch.float32 or d_final_state_bhkv.shape != state_bhkv.shape:
            raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, "d_final_state must be float32 shaped like the state")
    new = lambda t: torch.empty(t.shape, device=t.device, dtype=torch.float32)
    grads = dict(d_q=new(q_bshk), d_k=new(k_bshk), d_v=new(v_bshv), d_erase=new(erase_bshK),
                 d_write=new(write_bshV), d_g=new(g_bshK) if has_gate else None, d_state=new(state_bhkv))
    bw = _abi.ChunkBwdArgs()
    bw.fwd = a
    bw.d_y = d_y_bshv.data_ptr()
    bw.d_state_final = None if d_final_state_bhkv is None else d_final_state_bhkv.data_ptr()
    for name, t in grads.items():
        setattr(bw, name, None if t is None else t.data_ptr())
    need = int(_abi.lib().dc_chunk_bwd_workspace_size(bw))
    if workspace is None:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=q_bshk.device)
    _check_tensor(workspace, "workspace")
    bw.workspace, bw.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    with torch.cuda.device(q_bshk.device):
        _raise(_abi.lib().dc_chunk_bwd(bw, torch.cuda.current_stream(q_bshk.device).cuda_stream), "dc_chunk_bwd")
    return (grads["d_q"], grads["d_k"], grads["d_v"], grads["d_erase"], grads["d_write"], grads["d_g"],
            grads["d_state"])


def out_norm(y_bshv: torch.Tensor, gate_bshv: Optional[torch.Tensor], weight: torch.Tensor, eps: float = 1e-5, *,
             out_dtype: Optional[torch.dtype] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The per-head output normalisation after the read-out, ``OutNorm::forward``
    (src/common/norm.rs:129-135), through ``dc_out_norm``: over the last axis
    (one head's ``head_v_dim`` values) of ``y``,
    ``y / sqrt(mean(y^2) + eps) * weight``, times ``silu(gate)`` when a gate is
    given (the gated form, burn-stack ``RmsNormGated``).  ``y`` and ``gate``
    share a dtype (float32 / bfloat16); ``weight`` is float32 ``[head_v_dim]``.
    Returns ``out`` (``y``'s shape, ``out_dtype`` or ``y``'s dtype); it may be
    ``y`` itself.  ``eps`` defaults to 1e-5 (Burn's RMSNorm default).
    """
    _check_tensor(y_bshv, "y")
    dv = y_bshv.shape[-1]
    if gate_bshv is not None:
        _check_tensor(gate_bshv, "gate")
        if gate_bshv.shape != y_bshv.shape:
            raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, f"gate has shape {tuple(gate_bshv.shape)}, want {tuple(y_bshv.shape)}")
    _check_tensor(weight, "weight")
    if weight.dtype != torch.float32 or tuple(weight.shape) != (dv,):
        raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, f"weight must be float32 [{dv}]")
    in_code = _same_dtype((y_bshv, gate_bshv), "y and gate")
    if out is None:
        out = torch.empty(y_bshv.shape, device=y_bshv.device, dtype=out_dtype or y_bshv.dtype)
    _check_tensor(out, "out")
    if out.shape != y_bshv.shape:
        raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, "out must be shaped like y")
    a = _abi.OutNormArgs()
    a.rows, a.dv = y_bshv.numel() // max(dv, 1), dv
    a.in_dtype, a.out_dtype, a.eps = in_code, _dtype_code(out, "out"), float(eps)
    a.y, a.weight, a.out = y_bshv.data_ptr(), weight.data_ptr(), out.data_ptr()
    a.gate = None if gate_bshv is None else gate_bshv.data_ptr()
    with torch.cuda.device(y_bshv.device):
        _raise(_abi.lib().dc_out_norm(a, torch.cuda.current_stream(y_bshv.device).cuda_stream), "dc_out_norm")
    return out


def qkv_prologue(x_bsw: torch.Tensor, heads: int, dk: int, dv: int, conv_weight: torch.Tensor,
                 conv_bias: Optional[torch.Tensor] = None, window_bwc: Optional[torch.Tensor] = None, *,
                 n_householder: int = 1, conv_silu: bool = True, qk_silu: bool = False, l2: bool = True,
                 out_dtype: Optional[torch.dtype] = None):
    """The front-end between the input projection and the core (``QkvProjection::forward`` / ``step``
    after ``in_proj``, src/common/qkv.rs:373-500) through ``dc_qkv_prologue``.

    ``x_bsw`` ``[B, S, >= C]`` holds the projection's ``[q | u k | u v]`` channels first (C = heads dk
    (1 + u) + u heads dv; a column slice of the whole projection is fine).  The causal depthwise short
    convolution (``conv_weight [C, K]``, ``conv_bias [C]`` or None) runs over its channels with the
    rolling window ``window_bwc [B, C, K]`` (None: zeros; src/common/conv.rs:81-160), then SiLU
    (``conv_silu``; else SiLU on v and, with ``qk_silu``, on q and k), then the L2 norm of q and k over
    each head (``l2``).  Returns ``(q [B, S, H, dk], k [B, S u, H, dk], v [B, S u, H, dv], next window)``;
    a single-token ``step`` is ``S = 1``.
    """
    _check_tensor(conv_weight, "conv_weight")
    if not isinstance(x_bsw, torch.Tensor) or not x_bsw.is_cuda:
        raise DeltaCoreError(_abi.DC_EDEVICE, "x must be a CUDA tensor")
    if x_bsw.dim() != 3 or x_bsw.stride(2) != 1 or x_bsw.stride(0) != x_bsw.shape[1] * x_bsw.stride(1):
        raise DeltaCoreError(_abi.DC_EINVAL_ARG, "x must be [B, S, W] with contiguous channels and tokens")
    b, s, _ = x_bsw.shape
    u = int(n_householder)
    c = heads * dk * (1 + u) + u * heads * dv
    if conv_weight.dtype != torch.float32 or conv_weight.dim() != 2 or conv_weight.shape[0] != c:
        raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, f"conv_weight must be float32 [{c}, K]")
    kk = conv_weight.shape[1]
    if conv_bias is not None:
        _check_tensor(conv_bias, "conv_bias")
        if conv_bias.dtype != torch.float32 or tuple(conv_bias.shape) != (c,):
            raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, f"conv_bias must be float32 [{c}]")
    if window_bwc is not None:
        _check_tensor(window_bwc, "window")
        if window_bwc.dtype != torch.float32 or tuple(window_bwc.shape) != (b, c, kk):
            raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, f"window must be float32 [{b}, {c}, {kk}]")
    odt = out_dtype or x_bsw.dtype
    dev = x_bsw.device
    q = torch.empty(b, s, heads, dk, device=dev, dtype=odt)
    k = torch.empty(b, s * u, heads, dk, device=dev, dtype=odt)
    v = torch.empty(b, s * u, heads, dv, device=dev, dtype=odt)
    nxt = torch.empty(b, c, kk, device=dev, dtype=torch.float32)
    a = _abi.PrologueArgs()
    a.batch, a.seq, a.heads, a.dk, a.dv = b, s, heads, dk, dv
    a.n_householder, a.conv_kernel = u, kk
    a.in_dtype, a.out_dtype = _dtype_code(x_bsw, "x"), _dtype_code(q, "out")
    a.flags = ((_abi.DC_PROLOGUE_CONV_SILU if conv_silu else 0) | (_abi.DC_PROLOGUE_QK_SILU if qk_silu else 0)
               | (_abi.DC_PROLOGUE_L2 if l2 else 0))
    a.x_stride = x_bsw.stride(1)
    a.x, a.conv_weight = x_bsw.data_ptr(), conv_weight.data_ptr()
    a.conv_bias = None if conv_bias is None else conv_bias.data_ptr()
    a.window_in = None if window_bwc is None else window_bwc.data_ptr()
    a.window_out = nxt.data_ptr()
    a.q, a.k, a.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    with torch.cuda.device(dev):
        _raise(_abi.lib().dc_qkv_prologue(a, torch.cuda.current_stream(dev).cuda_stream), "dc_qkv_prologue")
    return q, k, v, nxt


def _gates(x: torch.Tensor, kind: int, cols_out, group=1, scale=1.0, lo=0.0, hi=0.0, bias=None, a_log=None):
    """dc_gates over the last axis of x (a [.., cols] column slice; rows contiguous in the leading axes)."""
    if not isinstance(x, torch.Tensor) or not x.is_cuda:
        raise DeltaCoreError(_abi.DC_EDEVICE, "x must be a CUDA tensor")
    cols = x.shape[-1]
    rows = x.numel() // max(cols, 1)
    x2 = x.reshape(rows, cols) if x.dim() != 2 else x
    if x2.stride(1) != 1 or (rows > 1 and x2.stride(0) < cols):
        raise DeltaCoreError(_abi.DC_EINVAL_ARG, "x must have contiguous columns and one row stride")
    for t, name in ((bias, "bias"), (a_log, "a_log")):
        if t is not None:
            _check_tensor(t, name)
            if t.dtype != torch.float32:
                raise DeltaCoreError(_abi.DC_EUNSUPPORTED_DTYPE, f"{name} must be float32")
    out = torch.empty(tuple(x.shape[:-1]) + tuple(cols_out), device=x.device, dtype=torch.float32)
    a = _abi.GateArgs()
    a.rows, a.cols, a.x_stride = rows, cols, x2.stride(0) if rows > 1 else cols
    a.kind, a.in_dtype, a.group = kind, _dtype_code(x, "x"), group
    a.scale, a.lo, a.hi = scale, lo, hi
    a.x, a.out = x2.data_ptr(), out.data_ptr()
    a.bias = None if bias is None else bias.data_ptr()
    a.a_log = None if a_log is None else a_log.data_ptr()
    with torch.cuda.device(x.device):
        _raise(_abi.lib().dc_gates(a, torch.cuda.current_stream(x.device).cuda_stream), "dc_gates")
    return out


def write_gate(raw: torch.Tensor, doubled: bool = False) -> torch.Tensor:
    """The write gates of ``squash_write`` (src/common/qkv.rs:333-368) through ``dc_gates``:
    ``sigmoid(raw)``, times 2 for the erase gate under ``allow_neg_eigval``.  ``raw`` may be a column
    slice of the projection; returns float32 of ``raw``'s shape."""
    return _gates(raw, _abi.DC_GATE_WRITE, (raw.shape[-1],), scale=2.0 if doubled else 1.0)


def head_log_decay(dt_raw: torch.Tensor, dt_bias: torch.Tensor, a_log: torch.Tensor,
                   dt_limit=(0.0, 6.5504e4)) -> torch.Tensor:
    """``ForgetGate::log_decay`` (src/common/gate.rs:51-59) through ``dc_gates``:
    ``clamp(softplus(dt_raw + dt_bias), *dt_limit) * -exp(a_log)`` over the last axis (heads)."""
    h = dt_raw.shape[-1]
    if tuple(dt_bias.shape) != (h,) or tuple(a_log.shape) != (h,):
        raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, f"dt_bias and a_log must be [{h}]")
    return _gates(dt_raw, _abi.DC_GATE_HEAD_DECAY, (h,), lo=float(dt_limit[0]), hi=float(dt_limit[1]),
                  bias=dt_bias, a_log=a_log)


def channel_log_decay(dt: torch.Tensor, dt_bias: torch.Tensor, a_log: torch.Tensor, head_k_dim: int,
                      lower_bound: float) -> torch.Tensor:
    """``ChannelForgetGate::log_decay`` (src/common/gate.rs:178-196) through ``dc_gates``, on its ``up``
    projection's output ``dt [.., heads * head_k_dim]``: ``lower_bound * sigmoid((dt + dt_bias) *
    exp(a_log[head]))``, returned as float32 ``[.., heads, head_k_dim]``."""
    c = dt.shape[-1]
    if c % head_k_dim or tuple(dt_bias.shape) != (c,) or tuple(a_log.shape) != (c // head_k_dim,):
        raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, "dt_bias must be [heads * head_k_dim], a_log [heads]")
    return _gates(dt, _abi.DC_GATE_CHANNEL_DECAY, (c // head_k_dim, head_k_dim), group=head_k_dim,
                  scale=float(lower_bound), bias=dt_bias, a_log=a_log)


class DeltaChunkFunction(torch.autograd.Function):
    """The custom autodiff node (src/delta/chunk_recalculated/backward.rs:30-265): the forward
    keeps only its leaf inputs, and the backward recomputes what it needs from them.

    ``y, final_state = DeltaChunkFunction.apply(q, k, v, erase, write, g, state, has_gate,
    chunk_len, scale, n_householder)``; gradients flow to every tensor input (``g`` when
    ``has_gate``).  y is float32."""

    @staticmethod
    def forward(ctx, q, k, v, erase, write, g, state, has_gate, chunk_len, scale, n_householder=1):
        y, s_out = delta_chunk_recalculated(q, k, v, erase, write, g, state, has_gate, chunk_len, scale,
                                            n_householder=n_householder, out_dtype=torch.float32)
        ctx.save_for_backward(q, k, v, erase, write, g if has_gate else None, state)
        ctx.cfg = (has_gate, chunk_len, scale, n_householder)
        return y, s_out

    @staticmethod
    def backward(ctx, d_y, d_state):
        q, k, v, erase, write, g, state = ctx.saved_tensors
        has_gate, chunk_len, scale, u = ctx.cfg
        d_y = torch.zeros_like(v[:, :q.shape[1]], dtype=torch.float32) if d_y is None else d_y.float().contiguous()
        d_state = None if d_state is None else d_state.float().contiguous()
        dq, dk, dv, de, dw, dg, ds = delta_chunk_recalculated_backward(
            d_y, d_state, q, k, v, erase, write, g, state, has_gate, chunk_len, scale, n_householder=u)
        cast = lambda grad, like: None if grad is None else grad.to(like.dtype)
        return (cast(dq, q), cast(dk, k), cast(dv, v), cast(de, erase), cast(dw, write),
                cast(dg, g) if has_gate else None, cast(ds, state), None, None, None, None)


def _check_host_tensor(t: torch.Tensor, what: str) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{what} must be a torch.Tensor")
    if t.device.type != "cpu":
        raise DeltaCoreError(_abi.DC_EINVAL_ARG, f"{what} is on {t.device}: this entry point takes host tensors")
    if not t.is_contiguous():
        raise DeltaCoreError(_abi.DC_EINVAL_ARG, f"{what} must be contiguous")


def delta_chunk_host_scratch_size(q_bshk, k_bshk, v_bshv, erase_bshK, write_bshV, g_bshK, state_bhkv,
                                  has_gate: bool, chunk_len: int, scale: float, *, n_householder: int = 1,
                                  out_dtype: Optional[torch.dtype] = None, force_simt: bool = False,
                                  force_split: bool = False) -> int:
    """Bytes of device scratch :func:`delta_chunk_recalculated_host` needs for
    these host tensors (``dc_chunk_fwd_host_scratch_size``)."""
    a = _chunk_args(q_bshk, k_bshk, v_bshv, erase_bshK, write_bshV, g_bshK, state_bhkv, has_gate, chunk_len,
                    scale, n_householder, out_dtype, force_simt, False, force_split, None, None,
                    _check_host_tensor, lambda shape, dt: torch.empty(shape, dtype=dt))[0]
    return int(_abi.lib().dc_chunk_fwd_host_scratch_size(a))


def delta_chunk_recalculated_host(q_bshk, k_bshk, v_bshv, erase_bshK, write_bshV, g_bshK, state_bhkv,
                                  has_gate: bool, chunk_len: int, scale: float, *, n_householder: int = 1,
                                  out_dtype: Optional[torch.dtype] = None, force_simt: bool = False,
                                  force_split: bool = False, device=None, scratch: Optional[torch.Tensor] = None,
                                  y_out: Optional[torch.Tensor] = None, state_out: Optional[torch.Tensor] = None,
                                  synchronize: bool = True):
    """:func:`delta_chunk_recalculated` on HOST tensors (pinned for full PCIe
    speed) through ``dc_chunk_fwd_host``: the batch is streamed through the
    GPU in slices of whole sequences, copies in both directions overlapping
    the kernels.  Outputs are host tensors (pinned when allocated here).
    ``scratch`` is a uint8 CUDA tensor of ``dc_chunk_fwd_host_scratch_size``
    bytes to reuse (allocated per call otherwise).  With ``synchronize=False``
    the call returns once the work is queued on the device's current stream;
    the outputs are complete when that stream has drained.
    """
    dev = torch.device(device if device is not None else "cuda")
    pin = lambda shape, dt: torch.empty(shape, dtype=dt, pin_memory=True)
    a, y, s_out = _chunk_args(q_bshk, k_bshk, v_bshv, erase_bshK, write_bshV, g_bshK, state_bhkv, has_gate,
                              chunk_len, scale, n_householder, out_dtype, force_simt, False, force_split,
                              y_out, state_out, _check_host_tensor, pin)
    need = int(_abi.lib().dc_chunk_fwd_host_scratch_size(a))
    if scratch is None:
        scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    _check_tensor(scratch, "scratch")
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        _raise(_abi.lib().dc_chunk_fwd_host(a, scratch.data_ptr(), scratch.numel(), stream.cuda_stream),
               "dc_chunk_fwd_host")
        if synchronize:
            stream.synchronize()
    return y, s_out


def delta_step(q_bhk, k_bhk, v_bhv, erase_bhK, write_bhV, g_bhK, state_bhkv, scale: float, *,
               n_householder: int = 1, out_dtype: Optional[torch.dtype] = None, force_simt: bool = False,
               y_out: Optional[torch.Tensor] = None, state_out: Optional[torch.Tensor] = None):
    """One delta-rule tick for all heads (src/delta/recurrent.rs:41-99).

    Shapes: q [b, h, dk]; k [b, h, dk] (or [b, u, h, dk] with ``n_householder=u``);
    v [b, h, dv] (or [b, u, h, dv]); erase [b, h, 1|dk]; write [b, h, 1|dv];
    g ``None`` or [b, h, 1|dk]; state [b, h, dk, dv] float32.
    Returns ``(y [b, h, dv], next_state)``; pass ``state_out=state_bhkv`` to
    update the state in place.
    """
    u = int(n_householder)
    for name, t in dict(q=q_bhk, k=k_bhk, v=v_bhv, erase=erase_bhK, write=write_bhV, state=state_bhkv).items():
        _check_tensor(t, name)
    if g_bhK is not None:
        _check_tensor(g_bhK, "g")
    if q_bhk.dim() != 3:
        raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, "q must be [batch, nheads, head_k_dim]")
    b, h, dk = q_bhk.shape
    lift = lambda t: t.unsqueeze(1) if t.dim() == 3 else t  # [b, h, .] -> [b, 1, h, .]
    k4, v4, e4, w4 = (lift(t) for t in (k_bhk, v_bhv, erase_bhK, write_bhV))
    dv = v4.shape[3]
    if tuple(k4.shape) != (b, u, h, dk) or tuple(v4.shape[:3]) != (b, u, h):
        raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, "k / v do not match q and n_householder")
    if tuple(state_bhkv.shape) != (b, h, dk, dv):
        raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, f"state has shape {tuple(state_bhkv.shape)}")
    for name, t, full in (("erase", e4, dk), ("write", w4, dv)):
        if tuple(t.shape[:3]) != (b, u, h):
            raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, f"{name} has shape {tuple(t.shape)}")
        if t.shape[3] not in (1, full):
            raise DeltaShapeError(_abi.DC_EINVAL_WIDTH, f"{name}: last axis must be 1 or {full}")
    if g_bhK is not None:
        if tuple(g_bhK.shape[:2]) != (b, h) or g_bhK.shape[2] not in (1, dk):
            raise DeltaShapeError(_abi.DC_EINVAL_WIDTH, f"forget gate has shape {tuple(g_bhK.shape)}")
    if state_bhkv.dtype != torch.float32:
        raise DeltaCoreError(_abi.DC_EUNSUPPORTED_DTYPE, "the state is float32")
    in_dt = _same_dtype((q_bhk, k_bhk, v_bhv), "q, k, v")
    gate_dt = _same_dtype((erase_bhK, write_bhV, g_bhK), "erase, write, g")
    y = y_out if y_out is not None else torch.empty((b, h, dv), device=q_bhk.device,
                                                    dtype=out_dtype or q_bhk.dtype)
    s_out = state_out if state_out is not None else torch.empty_like(state_bhkv)
    a = _abi.StepArgs()
    a.batch, a.heads, a.dk, a.dv = b, h, dk, dv
    a.n_householder = u
    a.erase_w, a.write_w = e4.shape[3], w4.shape[3]
    a.g_w = 0 if g_bhK is None else g_bhK.shape[2]
    a.in_dtype, a.gate_dtype, a.out_dtype = in_dt, gate_dt, _dtype_code(y, "y")
    a.flags = _abi.DC_FLAG_FORCE_SIMT if force_simt else 0  # the per-tile kernel instead of the streaming one
    a.scale = float(scale)
    a.q, a.k, a.v = q_bhk.data_ptr(), k_bhk.data_ptr(), v_bhv.data_ptr()
    a.erase, a.write = erase_bhK.data_ptr(), write_bhV.data_ptr()
    a.g = None if g_bhK is None else g_bhK.data_ptr()
    a.state_in, a.y, a.state_out = state_bhkv.data_ptr(), y.data_ptr(), s_out.data_ptr()
    with torch.cuda.device(q_bhk.device):
        stream = torch.cuda.current_stream(q_bhk.device).cuda_stream
        _raise(_abi.lib().dc_step(a, stream), "dc_step")
    san(y, "y")  # recurrent.rs:96-97
    san(s_out, "next state")
    return y, s_out


@dataclass
class DeltaInput:
    """Everything the delta-rule core consumes (src/delta/path.rs:120-141).

    q/k arrive activated and L2-normalised but not scaled; gates arrive
    squashed into their ranges; ``scale=None`` means 1/sqrt(head_k_dim)."""
    q_bshk: torch.Tensor
    k_bshk: torch.Tensor
    v_bshv: torch.Tensor
    erase_bshK: torch.Tensor
    write_bshV: torch.Tensor
    g_bshK: Optional[torch.Tensor]
    state_bhkv: torch.Tensor
    scale: Optional[float] = None
    n_householder: int = 1

    def dims(self):
        """(batch, sequence, nheads, head_k_dim, head_v_dim) — path.rs:154-158."""
        b, s, h, dk = self.q_bshk.shape
        return b, s, h, dk, self.v_bshv.shape[3]

    def resolved_scale(self) -> float:
        """path.rs:161-165."""
        return self.scale if self.scale is not None else 1.0 / math.sqrt(self.q_bshk.shape[3])

    def has_channel_decay(self) -> bool:
        """path.rs:170-172."""
        return self.g_bshK is not None and self.g_bshK.shape[3] > 1

    def sanity(self) -> None:
        """Shape and width checks (path.rs:177-208), then the NaN / Inf guard over
        every input (path.rs:198-207), which runs only when switched on
        (:func:`set_sanity_checks`), as the reference's runs only under its
        check-nan / check-inf features."""
        b, s, h, dk, dv = self.dims()
        u = self.n_householder
        if s < 1:
            raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, "sequence length must be at least 1")
        if tuple(self.k_bshk.shape) != (b, s * u, h, dk):
            raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, "k does not match q")
        if tuple(self.v_bshv.shape[:3]) != (b, s * u, h):
            raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, "v does not match q")
        if tuple(self.state_bhkv.shape) != (b, h, dk, dv):
            raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, "state does not match q / v")
        gates = [("erase gate", self.erase_bshK, s * u, dk), ("write gate", self.write_bshV, s * u, dv)]
        if self.g_bshK is not None:
            gates.append(("forget gate", self.g_bshK, s, dk))
        for what, t, rows, full in gates:
            if tuple(t.shape[:3]) != (b, rows, h):
                raise DeltaShapeError(_abi.DC_EINVAL_SHAPE, what)
            if t.shape[3] not in (1, full):
                raise DeltaShapeError(_abi.DC_EINVAL_WIDTH,
                                      f"{what}: last axis must be 1 or {full}, got {t.shape[3]}")
        for what, t in (("q", self.q_bshk), ("k", self.k_bshk), ("v", self.v_bshv), ("erase gate", self.erase_bshK),
                        ("write gate", self.write_bshV), ("state", self.state_bhkv), ("forget gate", self.g_bshK)):
            san(t, what)

    def run(self, path: DeltaPath = DeltaPath.default()):
        """Run the selected algorithm (path.rs:215-231); returns (y_bshv, final_state_bhkv)."""
        self.sanity()
        if path.kind != "recurrent":
            chunk_len = path.resolved_chunk_len()
            if chunk_len < 1:
                raise DeltaCoreError(_abi.DC_EINVAL_ARG, "chunk_len must be at least 1")
            return delta_chunk_recalculated(
                self.q_bshk, self.k_bshk, self.v_bshv, self.erase_bshK, self.write_bshV, self.g_bshK,
                self.state_bhkv, self.g_bshK is not None, chunk_len, self.resolved_scale(),
                n_householder=self.n_householder)
        return self.delta_recurrent()

    def delta_recurrent(self):
        """Unroll the fused step over the sequence (src/delta/recurrent.rs:107-142)."""
        return delta_chunk_recalculated(
            self.q_bshk, self.k_bshk, self.v_bshv, self.erase_bshK, self.write_bshV, self.g_bshK,
            self.state_bhkv, self.g_bshK is not None, 1, self.resolved_scale(),
            n_householder=self.n_householder, recurrent=True)

"""B200 (sm_100a) delta-rule core: a drop-in for burn-deltanet's src/delta path.

The package directory name is not a Python identifier; import it with
``importlib.import_module("burn-deltanet_b200")`` with the repository root on
``sys.path``.

* ``libdeltacore.so`` — the CUDA kernels behind the C ABI of include/deltacore.h
  (built in-tree by ``build.py``);
* :mod:`.core`     — the reference's interface (DeltaInput, DeltaPath, delta_step, ...)
  over that ABI, the custom backward (delta_chunk_recalculated_backward,
  DeltaChunkFunction), and the block's kernels on either side of the core: the
  front-end after the input projection (qkv_prologue, write_gate,
  head_log_decay, channel_log_decay) and the output norm (out_norm);
* :mod:`.sharding` — batch x head partitioning across the GPUs of one node.
"""
from . import _abi
from .core import (
    DeltaChunkFunction,
    DeltaCoreError,
    DeltaInput,
    DeltaNonFiniteError,
    DeltaPath,
    DeltaShapeError,
    TriSolve,
    beta_gates,
    chunk_out_norm_is_fused,
    delta_chunk_host_scratch_size,
    delta_chunk_recalculated,
    delta_chunk_recalculated_backward,
    delta_chunk_recalculated_host,
    delta_chunk_recalculated_out_norm,
    delta_step,
    out_norm,
    qkv_prologue,
    write_gate,
    head_log_decay,
    channel_log_decay,
    san,
    set_sanity_checks,
)

__all__ = [
    "DeltaChunkFunction", "DeltaCoreError", "DeltaInput", "DeltaNonFiniteError", "DeltaPath", "DeltaShapeError",
    "TriSolve", "san", "set_sanity_checks",
    "beta_gates", "delta_chunk_host_scratch_size", "delta_chunk_recalculated", "delta_chunk_recalculated_backward",
    "delta_chunk_recalculated_host", "delta_chunk_recalculated_out_norm", "chunk_out_norm_is_fused", "delta_step", "library_path", "out_norm", "qkv_prologue", "write_gate", "head_log_decay", "channel_log_decay",
]


def library_path() -> str:
    return _abi.LIB_PATH

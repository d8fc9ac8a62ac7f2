"""CPU oracle for the per-head output normalisation.

TEST INFRASTRUCTURE ONLY (see the package docstring): the parity checker of
``dc_out_norm``.

The reference's ``OutNorm`` (src/common/norm.rs:106-144) wraps burn-stack's
``RmsNormGated`` and ``RmsNorm`` (burn-stack rev 984d42d3, Cargo.toml:52).
That crate is not vendored in the reference tree, so this restates the form
norm.rs:106-113 documents: per (batch, token, head) row of y over its
``head_v_dim`` values,

    rms(y) = y / sqrt(mean(y^2) + eps)
    gated:   rms(y) * weight * silu(gate),   silu(x) = x * sigmoid(x)
    plain:   rms(y) * weight

in float64.  The plain form is pinned to ``torch.nn.functional.rms_norm`` by
tests/test_oracle_out_norm.py.  burn-stack's default epsilon is not in the
reference tree, so the callers pass it.  Parity with burn-stack itself is
therefore anchored on this documented form, not on burn-stack's source.
"""
from __future__ import annotations

import numpy as np


def out_norm(y, gate, weight, eps):
    """OutNorm::forward (norm.rs:129-135): y [..., dv], gate None or like y, weight [dv]."""
    y = np.asarray(y, dtype=np.float64)
    w = np.asarray(weight, dtype=np.float64)
    out = y / np.sqrt((y * y).mean(axis=-1, keepdims=True) + float(eps)) * w
    if gate is not None:
        g = np.asarray(gate, dtype=np.float64)
        out = out * (g / (1.0 + np.exp(-g)))
    return out

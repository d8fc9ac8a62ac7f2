"""CPU oracle for the front-end between the fused input projection and the delta-rule core.

TEST INFRASTRUCTURE ONLY (see the package docstring): the parity checker of
``dc_qkv_prologue``.

Restates, in float64, the part of ``QkvProjection::forward`` / ``step``
(src/common/qkv.rs:373-440, 447-500) that runs after ``in_proj``, on the
``[q | u k | u v]`` channel segment of the projection:

* the causal depthwise short convolution with its rolling window
  (src/common/conv.rs:81-118 forward, 124-160 step): the input is left-padded
  with the window's newest ``K - 1`` columns, ``y[c, t] = bias[c] +
  sum_j w[c, j] x_pad[c, t + j]``, and the next window is the last ``K``
  columns of the padded input; then the convolution's activation (SiLU or
  none, conv.rs:26-46);
* the split into q ``[B, S, H, dk]``, k ``[B, S u, H, dk]``, v
  ``[B, S u, H, dv]`` (a reshape: micro-step m of token t is row t u + m);
* when the activation is not the convolution's: q / k through the q/k
  activation (src/common/norm.rs QkActivation: identity or SiLU) and v
  through SiLU (qkv.rs:405-413);
* the q / k normalisation over the head axis: ``x / sqrt(sum x^2 + 1e-6)``
  (norm.rs:83-90, L2_EPS) or none.

``step`` is the same computation on a one-token sequence (conv.rs:124-160
evaluates the filter on [window[1:], x], the forward's padded form at S = 1).
"""
from __future__ import annotations

import numpy as np

L2_EPS = 1e-6


def _silu(x):
    return x / (1.0 + np.exp(-x))


def qkv_prologue(x, heads, dk, dv, u, weight, bias, window, conv_silu=True, qk_silu=False, l2=True):
    """x [B, S, C] (C = heads dk (1 + u) + u heads dv), weight [C, K], bias None or [C], window None or
    [B, C, K].  Returns q [B, S, H, dk], k [B, S u, H, dk], v [B, S u, H, dv], next window [B, C, K]."""
    x = np.asarray(x, dtype=np.float64)
    w = np.asarray(weight, dtype=np.float64)
    b_, s, c = x.shape
    kk = w.shape[1]
    win = np.zeros((b_, c, kk)) if window is None else np.asarray(window, dtype=np.float64)
    pad = np.concatenate([win[:, :, 1:], np.transpose(x, (0, 2, 1))], axis=2)  # [B, C, K - 1 + S]
    nxt = pad[:, :, s - 1:s - 1 + kk].copy()
    y = np.zeros((b_, c, s))
    for j in range(kk):
        y += w[None, :, j:j + 1] * pad[:, :, j:j + s]
    if bias is not None:
        y += np.asarray(bias, dtype=np.float64)[None, :, None]
    y = np.transpose(y, (0, 2, 1))  # [B, S, C]
    if conv_silu:
        y = _silu(y)
    kd = heads * dk
    q = y[:, :, :kd].reshape(b_, s, heads, dk)
    k = y[:, :, kd:kd + u * kd].reshape(b_, s * u, heads, dk)
    v = y[:, :, kd + u * kd:].reshape(b_, s * u, heads, dv)
    if not conv_silu:
        if qk_silu:
            q, k = _silu(q), _silu(k)
        v = _silu(v)
    if l2:
        q = q / np.sqrt((q * q).sum(-1, keepdims=True) + L2_EPS)
        k = k / np.sqrt((k * k).sum(-1, keepdims=True) + L2_EPS)
    return q, k, v, nxt

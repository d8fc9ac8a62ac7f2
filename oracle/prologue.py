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


# ---------------------------------------------------------------------------------------------------
# The gate producers of the front-end (float64).
# ---------------------------------------------------------------------------------------------------
def softplus(x):
    """log(1 + e^x), in the overflow-free form max(x, 0) + log1p(e^-|x|) (burn-stack's ``softplus``,
    rev 984d42d3, is not vendored in the reference tree; this is the function's definition)."""
    x = np.asarray(x, dtype=np.float64)
    return np.maximum(x, 0.0) + np.log1p(np.exp(-np.abs(x)))


def write_gate(raw, doubled):
    """``squash_write`` (src/common/qkv.rs:333-368): sigma(raw), times 2 for the erase gate under
    ``allow_neg_eigval`` (``doubled``)."""
    raw = np.asarray(raw, dtype=np.float64)
    return (2.0 if doubled else 1.0) / (1.0 + np.exp(-raw))


def head_log_decay(dt_raw, dt_bias, a_log, dt_limit=(0.0, 6.5504e4)):
    """``ForgetGate::log_decay`` (src/common/gate.rs:51-59): g = clamp(softplus(dt + b), lo, hi) * -e^a,
    the per-head parameters broadcast over the last axis (heads)."""
    dt = softplus(np.asarray(dt_raw, dtype=np.float64) + np.asarray(dt_bias, dtype=np.float64))
    return np.clip(dt, dt_limit[0], dt_limit[1]) * -np.exp(np.asarray(a_log, dtype=np.float64))


def channel_log_decay(dt, dt_bias, a_log, head_k_dim, lower_bound):
    """``ChannelForgetGate::log_decay`` (src/common/gate.rs:178-196) after its ``up`` projection: the
    channels [.., heads * head_k_dim] plus the bias, split per head, g = lower_bound *
    sigmoid(dt * e^{a_h}).  Returns [.., heads, head_k_dim]."""
    dt = np.asarray(dt, dtype=np.float64) + np.asarray(dt_bias, dtype=np.float64)
    shape = dt.shape[:-1] + (-1, head_k_dim)
    dt = dt.reshape(shape)
    slope = np.exp(np.asarray(a_log, dtype=np.float64))[:, None]
    return float(lower_bound) / (1.0 + np.exp(-dt * slope))

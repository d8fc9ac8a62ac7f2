"""CPU oracle for the backward of the delta-rule core.

TEST INFRASTRUCTURE ONLY (see the package docstring): the parity checker of
``dc_chunk_bwd``.

The gradients the reference's custom autodiff node returns
(src/delta/chunk_recalculated/combined_backward.rs:72-190, ``DeltaChunkGrads``)
are the derivatives of L = <y, d_y> + <final_state, d_state_final> through the
forward.  The reference differentiates its chunkwise forward; the chunkwise
forward equals the recurrence (src/delta/recurrent.rs:41-142, the definition
the reference's tests pin every path to), so this oracle differentiates the
recurrence, step by step in float64:

    S-  = diag(alpha_t) S_{t-1}        (alpha = e^g on the key axis; 1 ungated)
    u_t = w_t * v_t - S-^T (b_t * k_t)
    S_t = S- + k_t u_t^T
    y_t = S_t^T (s q_t)

back to front, carrying dS.  n_householder > 1 runs on the folded sequence
(q on the last micro-step, g on the first; src/delta_product/delta_product.rs:
178-228) and unfolds the q and g gradients.  ``tests/test_oracle_backward.py``
checks this against torch autograd of the same recurrence.
"""
from __future__ import annotations

import numpy as np


def _expand(x, width):
    """[..., 1 | width] -> [..., width] (the gates' broadcast width)."""
    return np.broadcast_to(x, x.shape[:-1] + (width,))


def _reduce(g, width):
    """A full-width gradient summed back onto a gate of width 1."""
    return g.sum(axis=-1, keepdims=True) if width == 1 else g


def recurrent_backward(q, k, v, erase, write, g, state, d_y, d_state_final=None, scale=None,
                       n_householder=1):
    """Gradients of L = <y, d_y> + <S_final, d_state_final> for one forward call.

    Shapes as the forward: q [b, t, h, dk]; k [b, t*u, h, dk]; v [b, t*u, h, dv];
    erase [b, t*u, h, 1|dk]; write [b, t*u, h, 1|dv]; g None or [b, t, h, 1|dk];
    state [b, h, dk, dv]; d_y [b, t, h, dv]; d_state_final None or like state.
    Returns dict(d_q, d_k, d_v, d_erase, d_write, d_g (None if ungated), d_state).
    """
    q, k, v = (np.asarray(x, dtype=np.float64) for x in (q, k, v))
    erase, write = np.asarray(erase, dtype=np.float64), np.asarray(write, dtype=np.float64)
    state = np.asarray(state, dtype=np.float64)
    d_y = np.asarray(d_y, dtype=np.float64)
    u = int(n_householder)
    b, t, h, dk = q.shape
    dv = v.shape[3]
    n = t * u
    s = 1.0 / np.sqrt(dk) if scale is None else float(scale)
    ew, ww = erase.shape[3], write.shape[3]
    gw = 0 if g is None else np.asarray(g).shape[3]
    # the folded sequence: q and dy on the last micro-step, g on the first
    qf = np.zeros((b, n, h, dk))
    qf[:, u - 1::u] = q
    dyf = np.zeros((b, n, h, dv))
    dyf[:, u - 1::u] = d_y
    gf = None
    if gw:
        gf = np.zeros((b, n, h, gw))
        gf[:, 0::u] = np.asarray(g, dtype=np.float64)
    e_full, w_full = _expand(erase, dk), _expand(write, dv)

    # forward, keeping S- and u of every step
    S = state.copy()
    S_minus = np.empty((n, b, h, dk, dv))
    U = np.empty((n, b, h, dv))
    A = np.ones((n, b, h, dk))
    for i in range(n):
        if gw:
            A[i] = np.exp(_expand(gf[:, i], dk))
            S = A[i][..., None] * S
        S_minus[i] = S
        bk = e_full[:, i] * k[:, i]
        U[i] = w_full[:, i] * v[:, i] - np.einsum("bhij,bhi->bhj", S, bk)
        S = S + k[:, i][..., None] * U[i][:, :, None, :]

    # backward
    dS = np.zeros_like(state) if d_state_final is None else np.asarray(d_state_final, dtype=np.float64).copy()
    dqf = np.zeros((b, n, h, dk))
    dk_ = np.zeros((b, n, h, dk))
    dv_ = np.zeros((b, n, h, dv))
    de = np.zeros((b, n, h, dk))
    dw = np.zeros((b, n, h, dv))
    dgf = np.zeros((b, n, h, dk))
    for i in range(n - 1, -1, -1):
        Sm, ui = S_minus[i], U[i]
        St = Sm + k[:, i][..., None] * ui[:, :, None, :]
        dyi = dyf[:, i]
        dqf[:, i] = s * np.einsum("bhij,bhj->bhi", St, dyi)
        dS = dS + (s * qf[:, i])[..., None] * dyi[:, :, None, :]
        du = np.einsum("bhij,bhi->bhj", dS, k[:, i])
        r = np.einsum("bhij,bhj->bhi", Sm, du)
        dk_[:, i] = np.einsum("bhij,bhj->bhi", dS, ui) - e_full[:, i] * r
        de[:, i] = -k[:, i] * r
        dv_[:, i] = w_full[:, i] * du
        dw[:, i] = v[:, i] * du
        bk = e_full[:, i] * k[:, i]
        dS = dS - bk[..., None] * du[:, :, None, :]
        if gw:
            dgf[:, i] = (dS * Sm).sum(axis=-1)
            dS = A[i][..., None] * dS

    d_g = None
    if gw:
        d_g = _reduce(dgf[:, 0::u], gw)
    return dict(d_q=dqf[:, u - 1::u], d_k=dk_, d_v=dv_, d_erase=_reduce(de, ew), d_write=_reduce(dw, ww),
                d_g=d_g, d_state=dS)

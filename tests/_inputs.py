"""Seeded input generators shared by the tests and the benchmark.

Two families of recipes:

* ``random_raw`` / ``constant_raw`` — the reference's own test inputs
  (src/delta/tests.rs:49-139 and :373-417): q and k L2-normalised N(0,1),
  v ~ N(0,1), erase ~ U(0.05, beta_max), write = erase (per head) or
  U(0.05, 1) (per channel), g ~ U(-0.5, -0.01), state zero or N(0, 0.2).
  The reference seeds nothing; these are seeded.
* ``config_inputs`` — the benchmark configurations' recipes (gates
  ``-exp(a)*softplus(x)`` with ``a ~ U(0, ln 16)``, beta = sigmoid or
  2*sigmoid, ...), usable at reduced sizes for parity tests.

All arrays are float64 numpy in the reference's layouts.
"""
from __future__ import annotations

import numpy as np

L2_EPS = 1e-6  # src/common/norm.rs:83


def l2_normalize(x):
    """x / sqrt(sum(x^2) + 1e-6) over the last axis (src/common/norm.rs:86-90)."""
    return x / np.sqrt((x * x).sum(-1, keepdims=True) + L2_EPS)


def softplus(x):
    return np.logaddexp(0.0, x)


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def random_raw(rng, batch, seq, heads, dk, dv, beta_max=0.95, gated=True, random_state=False,
               channel=False):
    q = l2_normalize(rng.standard_normal((batch, seq, heads, dk)))
    k = l2_normalize(rng.standard_normal((batch, seq, heads, dk)))
    v = rng.standard_normal((batch, seq, heads, dv))
    kw, vw = (dk, dv) if channel else (1, 1)
    erase = rng.uniform(0.05, beta_max, (batch, seq, heads, kw))
    write = rng.uniform(0.05, 1.0, (batch, seq, heads, vw)) if channel else erase.copy()
    g = rng.uniform(-0.5, -0.01, (batch, seq, heads, kw)) if gated else None
    state = (rng.normal(0.0, 0.2, (batch, heads, dk, dv)) if random_state
             else np.zeros((batch, heads, dk, dv)))
    return dict(q=q, k=k, v=v, erase=erase, write=write, g=g, state=state)


def constant_raw(rng, batch, seq, heads, dk, dv, beta, gated):
    """One direction per (batch, head) held for the whole sequence."""
    hold = lambda x: np.broadcast_to(x, (batch, seq, heads, x.shape[-1])).copy()
    q = hold(l2_normalize(rng.standard_normal((batch, 1, heads, dk))))
    k = hold(l2_normalize(rng.standard_normal((batch, 1, heads, dk))))
    v = hold(rng.standard_normal((batch, 1, heads, dv)))
    erase = np.full((batch, seq, heads, 1), beta)
    g = np.full((batch, seq, heads, 1), -0.05) if gated else None
    return dict(q=q, k=k, v=v, erase=erase, write=erase.copy(), g=g,
                state=np.zeros((batch, heads, dk, dv)))


def log_decay(rng, a_shape, x_shape):
    """log alpha = -exp(a) * softplus(x), a ~ U(0, ln 16) (fixed per head or
    per (head, channel)), x ~ N(0, 1) per token."""
    a = rng.uniform(0.0, np.log(16.0), a_shape)
    return -np.exp(a) * softplus(rng.standard_normal(x_shape))


def config_inputs(cfg, rng, batch, seq, heads, dk, dv, u=1, neg_eig=False):
    """The benchmark configurations' input recipes at any size.

    cfg 1 / 3 ("gdn"): scalar beta = sigmoid(N), per-head gate.
    cfg 2 ("deltanet"): beta = sigmoid(N) (2*sigmoid with neg_eig), no gate.
    cfg 4 ("deltaproduct"): u micro-steps with their own k, v, beta =
        2*sigmoid(N); per-head gate once per token; q once per token.
    cfg 5 ("gdn2"): per-channel erase b, write w = sigmoid(N); per-key-channel
        gate with a ~ U(0, ln 16) per (head, channel).
    k, v, erase, write carry seq*u rows; q and g carry seq rows.
    """
    su = seq * u
    q = l2_normalize(rng.standard_normal((batch, seq, heads, dk)))
    k = l2_normalize(rng.standard_normal((batch, su, heads, dk)))
    v = rng.standard_normal((batch, su, heads, dv))
    if cfg in ("gdn", 1, 3):
        beta = sigmoid(rng.standard_normal((batch, su, heads, 1)))
        erase, write = beta, beta.copy()
        g = log_decay(rng, (1, 1, heads, 1), (batch, seq, heads, 1))
    elif cfg in ("deltanet", 2):
        beta = sigmoid(rng.standard_normal((batch, su, heads, 1)))
        if neg_eig:
            beta = 2.0 * beta
        erase, write, g = beta, beta.copy(), None
    elif cfg in ("deltaproduct", 4):
        beta = 2.0 * sigmoid(rng.standard_normal((batch, su, heads, 1)))
        erase, write = beta, beta.copy()
        g = log_decay(rng, (1, 1, heads, 1), (batch, seq, heads, 1))
    elif cfg in ("gdn2", 5):
        erase = sigmoid(rng.standard_normal((batch, su, heads, dk)))
        write = sigmoid(rng.standard_normal((batch, su, heads, dv)))
        g = log_decay(rng, (1, 1, heads, dk), (batch, seq, heads, dk))
    else:
        raise ValueError(cfg)
    state = np.zeros((batch, heads, dk, dv))
    return dict(q=q, k=k, v=v, erase=erase, write=write, g=g, state=state)

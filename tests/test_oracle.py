"""The CPU oracle, pinned: the reference's golden vectors and the reference's
own known-answer and property tests (src/delta/tests.rs, src/delta/tri/tests.rs,
src/delta/chunk_recalculated/tests.rs), run on the float64 restatement.

The reference's tolerances are for float32 (1e-3 .. 1e-4); the float64
oracle is held to much tighter bounds where the mathematics is exact."""
import numpy as np
import pytest

import oracle
from _inputs import constant_raw, config_inputs, random_raw


def run(kind, raw, chunk_len=64, dtype=np.float64):
    args = (raw["q"], raw["k"], raw["v"], raw["erase"], raw["write"], raw["g"], raw["state"])
    if kind == "recurrent":
        return oracle.recurrent(*args, dtype=dtype)
    return oracle.chunk(*args, chunk_len=chunk_len, dtype=dtype)


# --------------------------------------------------------------------------
# Golden vectors: src/delta/tests.rs:533-568 and :760-812 (tolerance 1e-4).
# --------------------------------------------------------------------------
def golden_input(fx, kind):
    beta = fx["beta"][..., None]
    raw = dict(q=fx["q"], k=fx["k"], v=fx["v"], state=fx["state"])
    if kind == "ungated":
        raw.update(erase=beta, write=beta, g=None)
    elif kind == "gated":
        raw.update(erase=beta, write=beta, g=fx["g"][..., None])
    else:
        raw.update(erase=fx["b"], write=fx["w"], g=fx["gk"])
    return raw


@pytest.mark.parametrize("kind", ["ungated", "gated", "gdn2"])
@pytest.mark.parametrize("path", ["recurrent", 3, 4, 16, 64])
@pytest.mark.parametrize("dtype", [np.float64, np.float32])
def test_matches_the_reference_goldens(fla_golden, kind, path, dtype):
    raw = golden_input(fla_golden, kind)
    y, s = run("recurrent" if path == "recurrent" else "chunk", raw, path if path != "recurrent" else 1, dtype)
    want_y, want_s = fla_golden[f"{kind}_y"], fla_golden[f"{kind}_state"]
    assert np.abs(y - want_y).max() < 1e-6, "output differs from the reference golden"
    assert np.abs(s - want_s).max() < 1e-6, "final state differs from the reference golden"


# --------------------------------------------------------------------------
# chunk == recurrent: src/delta/tests.rs:300-337.
# --------------------------------------------------------------------------
@pytest.mark.parametrize(
    "b,s,h,dk,dv,L,beta_max,gated,rs",
    [
        (2, 16, 3, 8, 8, 8, 0.95, False, False),   # ungated
        (2, 16, 3, 8, 8, 8, 0.95, True, False),    # gated
        (2, 12, 2, 8, 16, 4, 0.95, True, True),    # carried state
        (2, 12, 2, 8, 8, 6, 1.95, True, True),     # negative eigenvalues
        (2, 13, 2, 8, 8, 8, 0.95, True, True),     # partial last chunk
        (1, 5, 1, 4, 4, 8, 0.95, False, False),    # partial, shorter than a chunk
        (2, 16, 2, 8, 16, 8, 0.95, True, True),    # dv != dk
    ],
)
def test_chunk_matches_recurrent(b, s, h, dk, dv, L, beta_max, gated, rs):
    raw = random_raw(np.random.default_rng(1), b, s, h, dk, dv, beta_max, gated, rs)
    y0, s0 = run("recurrent", raw)
    y1, s1 = run("chunk", raw, L)
    assert np.abs(y0 - y1).max() < 1e-9 and np.abs(s0 - s1).max() < 1e-9


def test_chunk_len_does_not_change_the_answer():
    raw = random_raw(np.random.default_rng(2), 2, 24, 2, 8, 8, 0.95, True, True)
    y0, s0 = run("chunk", raw, 4)
    for L in (1, 3, 6, 8, 12, 24, 32, 64):
        y, s = run("chunk", raw, L)
        assert np.abs(y - y0).max() < 1e-9 and np.abs(s - s0).max() < 1e-9, L


@pytest.mark.parametrize("beta,gated", [(0.9, False), (0.9, True), (1.8, True)])
def test_constant_input(beta, gated):
    """src/delta/tests.rs:423-460: the WY transform on a constant input."""
    raw = constant_raw(np.random.default_rng(3), 2, 128, 2, 8, 8, beta, gated)
    y0, s0 = run("recurrent", raw)
    for L in (16, 32, 48, 64, 128):
        y, s = run("chunk", raw, L)
        assert np.abs(y - y0).max() < 1e-8 and np.abs(s - s0).max() < 1e-8, L


def test_split_calls_match_a_single_call():
    """src/delta/tests.rs:465-494: streaming through the state."""
    raw = random_raw(np.random.default_rng(4), 2, 20, 2, 8, 8, 0.95, True, False)
    cut = lambda x, a, n: None if x is None else x[:, a:a + n]
    part = lambda a, n, st: {**{k: cut(raw[k], a, n) for k in ("q", "k", "v", "erase", "write", "g")}, "state": st}
    y_whole, s_whole = run("chunk", raw, 4)
    y_a, s_mid = run("chunk", part(0, 7, raw["state"]), 4)
    y_b, s_end = run("chunk", part(7, 13, s_mid), 4)
    assert np.abs(np.concatenate([y_a, y_b], 1) - y_whole).max() < 1e-9
    assert np.abs(s_end - s_whole).max() < 1e-9


def test_a_zero_gate_is_the_ungated_delta_rule():
    """src/delta/tests.rs:573-602."""
    raw = random_raw(np.random.default_rng(5), 2, 12, 2, 8, 8, 0.95, False, True)
    zero = dict(raw, g=np.zeros(raw["erase"].shape))
    for kind, L in (("recurrent", 1), ("chunk", 5)):
        y0, s0 = run(kind, raw, L)
        y1, s1 = run(kind, zero, L)
        assert np.abs(y0 - y1).max() < 1e-12 and np.abs(s0 - s1).max() < 1e-12


# --------------------------------------------------------------------------
# Channel gates (GDN-2): src/delta/tests.rs:614-756.
# --------------------------------------------------------------------------
@pytest.mark.parametrize(
    "b,s,h,dk,dv,L,beta_max,rs",
    [
        (2, 16, 3, 8, 8, 8, 0.95, False),
        (2, 12, 2, 8, 16, 4, 0.95, True),
        (2, 40, 2, 8, 8, 32, 0.95, True),   # across reference blocks
        (1, 37, 1, 4, 6, 16, 1.95, True),
        (2, 16, 2, 16, 8, 8, 0.95, True),   # dk > dv
    ],
)
def test_channel_chunk_matches_recurrent(b, s, h, dk, dv, L, beta_max, rs):
    raw = random_raw(np.random.default_rng(6), b, s, h, dk, dv, beta_max, True, rs, channel=True)
    y0, s0 = run("recurrent", raw)
    y1, s1 = run("chunk", raw, L)
    assert np.abs(y0 - y1).max() < 1e-9 and np.abs(s0 - s1).max() < 1e-9


def test_channel_chunk_len_does_not_change_the_answer():
    raw = random_raw(np.random.default_rng(7), 2, 24, 2, 8, 8, 0.95, True, True, channel=True)
    y0, s0 = run("recurrent", raw)
    for L in (1, 2, 3, 6, 8, 12, 16, 24, 32, 64):
        y, s = run("chunk", raw, L)
        assert np.abs(y - y0).max() < 1e-9 and np.abs(s - s0).max() < 1e-9, L


def test_broadcast_channel_gates_are_the_scalar_delta_rule():
    """src/delta/tests.rs:711-756."""
    raw = random_raw(np.random.default_rng(8), 2, 20, 2, 8, 12, 0.95, True, True)
    wide = dict(raw,
                erase=np.broadcast_to(raw["erase"], raw["erase"].shape[:3] + (8,)).copy(),
                write=np.broadcast_to(raw["write"], raw["write"].shape[:3] + (12,)).copy(),
                g=np.broadcast_to(raw["g"], raw["g"].shape[:3] + (8,)).copy())
    for kind, L in (("recurrent", 1), ("chunk", 8)):
        y0, s0 = run(kind, raw, L)
        y1, s1 = run(kind, wide, L)
        assert np.abs(y0 - y1).max() < 1e-12 and np.abs(s0 - s1).max() < 1e-12


def test_extreme_channel_gates_stay_finite_in_the_chunk_split():
    """BASELINE config 5's gates (-exp(a) softplus(x), a ~ U(0, ln 16)) exceed
    the reference's 48 exponent clamp over half a 16-row block
    (src/delta/decay.rs:41-49); its chunk path stays finite there, and the
    recurrent path is the exact definition parity is taken against."""
    raw = config_inputs(5, np.random.default_rng(9), 1, 96, 2, 16, 16)
    y0, s0 = run("recurrent", raw)
    y1, s1 = run("chunk", raw, 64)
    assert np.isfinite(y1).all() and np.isfinite(s1).all()
    assert np.isfinite(y0).all() and np.isfinite(s0).all()


# --------------------------------------------------------------------------
# The micro-step fold: src/delta_product/delta_product.rs:178-228.
# --------------------------------------------------------------------------
@pytest.mark.parametrize("u", [1, 2, 3])
def test_householder_fold_matches_manual_unroll(u):
    rng = np.random.default_rng(10 + u)
    raw = config_inputs(4, rng, 2, 7, 2, 8, 8, u=u)
    y, s = oracle.householder("recurrent", raw["q"], raw["k"], raw["v"], raw["erase"], raw["write"],
                              raw["g"], raw["state"], u)
    # Manual: step token by token, micro-step by micro-step.
    st = raw["state"].copy()
    ys = []
    for t in range(7):
        for m in range(u):
            r = t * u + m
            q = raw["q"][:, t] if m == u - 1 else np.zeros_like(raw["q"][:, t])
            g = raw["g"][:, t] if m == 0 else np.zeros_like(raw["g"][:, t])
            yt, st = oracle.step(q, raw["k"][:, r], raw["v"][:, r], raw["erase"][:, r], raw["write"][:, r], g, st,
                                 scale=1 / np.sqrt(8))
        ys.append(yt)
    assert np.abs(np.stack(ys, 1) - y).max() < 1e-12 and np.abs(st - s).max() < 1e-12
    yc, sc = oracle.householder("chunk", raw["q"], raw["k"], raw["v"], raw["erase"], raw["write"],
                                raw["g"], raw["state"], u, chunk_len=4)
    assert np.abs(yc - y).max() < 1e-9 and np.abs(sc - s).max() < 1e-9


# --------------------------------------------------------------------------
# Tri solve: src/delta/tri/tests.rs.
# --------------------------------------------------------------------------
@pytest.mark.parametrize("size", [1, 2, 3, 4, 5, 7, 8, 16, 32, 64, 128])
def test_blocked_inverts(size):
    n = np.tril(np.random.default_rng(size).normal(0, 0.3, (3, size, size)), -1)
    t = oracle.unit_lower_inverse(n)
    eye = np.eye(size)
    assert np.abs((eye - n) @ t - eye).max() < 1e-9
    assert np.abs(np.triu(t, 1)).max() == 0.0 and np.abs(np.diagonal(t, 0, 1, 2) - 1).max() < 1e-12


@pytest.mark.parametrize("size", [8, 16, 32, 64, 128])
@pytest.mark.parametrize("beta", [0.9, 1.0, 1.9])
def test_blocked_inverts_a_constant_key_chunk(size, beta):
    n = np.tril(np.full((size, size), -beta), -1)
    t = oracle.unit_lower_inverse(n)
    eye = np.eye(size)
    assert np.abs((eye - n) @ t - eye).max() < 1e-9
    assert np.abs(t).max() <= max(1.0, beta) + 1e-9


def test_float32_build_agrees_with_float64():
    raw = config_inputs(1, np.random.default_rng(11), 1, 200, 2, 32, 32)
    y0, s0 = run("recurrent", raw)
    y1, s1 = run("chunk", raw, 64, dtype=np.float32)
    scale = max(1.0, np.abs(y0).max())
    assert np.abs(y1 - y0).max() < 1e-4 * scale and np.abs(s1 - s0).max() < 1e-4 * max(1.0, np.abs(s0).max())

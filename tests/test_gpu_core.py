"""GPU parity: the CUDA kernels, called through the C ABI, against the CPU
oracle on the same seeded inputs — the reference's own test matrix
(src/delta/tests.rs, chunk_recalculated/tests.rs) plus the golden vectors.

Tolerances (written per test):
* float32 path: max |gpu - oracle| <= 1e-4 * max(1, max |oracle|) — the
  north star's "1e-4 relative" for the fp32 path.
* bf16 inputs with fp32 accumulation: the oracle runs on the same
  bf16-rounded inputs, so the float32 bound still applies to the CUDA-core
  kernels; the tensor-core kernel is held to 2e-2 max-abs.
"""
import importlib

import numpy as np
import pytest
import torch

import oracle
from _inputs import config_inputs, constant_raw, random_raw

pytestmark = pytest.mark.gpu
dn = importlib.import_module("burn-deltanet_b200")
abi = importlib.import_module("burn-deltanet_b200._abi")

F32_TOL = 1e-4


def to_dev(x, dtype=torch.float32):
    return None if x is None else torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


def rounded(x, dtype):
    """What the kernel actually reads: x cast to dtype, back in float64."""
    if x is None:
        return None
    return to_dev(x, dtype).double().cpu().numpy()


def rel_err(got, want):
    got = got.double().cpu().numpy() if isinstance(got, torch.Tensor) else got
    return np.abs(got - want).max() / max(1.0, np.abs(want).max())


def gpu_chunk(raw, chunk_len=64, u=1, in_dtype=torch.float32, gate_dtype=torch.float32, force_simt=False,
              scale=None):
    q, k, v = (to_dev(raw[n], in_dtype) for n in ("q", "k", "v"))
    e, w, g = (to_dev(raw[n], gate_dtype) for n in ("erase", "write", "g"))
    st = to_dev(raw["state"])
    sc = 1.0 / np.sqrt(raw["q"].shape[3]) if scale is None else scale
    y, s = dn.delta_chunk_recalculated(q, k, v, e, w, g, st, g is not None, chunk_len, sc, n_householder=u,
                                       out_dtype=torch.float32, force_simt=force_simt)
    torch.cuda.synchronize()
    return y, s


def oracle_run(raw, u=1, kind="recurrent", in_dtype=None, gate_dtype=None):
    r = dict(raw)
    if in_dtype is not None:
        for n in ("q", "k", "v"):
            r[n] = rounded(r[n], in_dtype)
    if gate_dtype is not None:
        for n in ("erase", "write", "g"):
            r[n] = rounded(r[n], gate_dtype)
    return oracle.householder(kind, r["q"], r["k"], r["v"], r["erase"], r["write"], r["g"], r["state"], u)


# --------------------------------------------------------------------------
# Golden vectors through the C ABI (src/delta/tests.rs:533-568, 760-812: 1e-4).
# --------------------------------------------------------------------------
@pytest.mark.parametrize("kind", ["ungated", "gated", "gdn2"])
@pytest.mark.parametrize("chunk_len", [3, 4, 16, 64])
def test_chunk_matches_the_reference_goldens(fla_golden, kind, chunk_len):
    fx = fla_golden
    beta = fx["beta"][..., None]
    raw = dict(q=fx["q"], k=fx["k"], v=fx["v"], state=fx["state"])
    if kind == "ungated":
        raw.update(erase=beta, write=beta, g=None)
    elif kind == "gated":
        raw.update(erase=beta, write=beta, g=fx["g"][..., None])
    else:
        raw.update(erase=fx["b"], write=fx["w"], g=fx["gk"])
    y, s = gpu_chunk(raw, chunk_len)
    assert np.abs(y.double().cpu().numpy() - fx[f"{kind}_y"]).max() < 1e-4
    assert np.abs(s.double().cpu().numpy() - fx[f"{kind}_state"]).max() < 1e-4


@pytest.mark.parametrize("kind", ["ungated", "gated", "gdn2"])
def test_recurrent_path_matches_the_reference_goldens(fla_golden, kind):
    fx = fla_golden
    beta = fx["beta"][..., None]
    if kind == "ungated":
        e, w, g = beta, beta, None
    elif kind == "gated":
        e, w, g = beta, beta, fx["g"][..., None]
    else:
        e, w, g = fx["b"], fx["w"], fx["gk"]
    inp = dn.DeltaInput(to_dev(fx["q"]), to_dev(fx["k"]), to_dev(fx["v"]), to_dev(e), to_dev(w), to_dev(g),
                        to_dev(fx["state"]))
    y, s = inp.run(dn.DeltaPath.Recurrent())
    assert np.abs(y.double().cpu().numpy() - fx[f"{kind}_y"]).max() < 1e-4
    assert np.abs(s.double().cpu().numpy() - fx[f"{kind}_state"]).max() < 1e-4


# --------------------------------------------------------------------------
# The reference's chunk == recurrent matrix (src/delta/tests.rs:300-337, 614-705).
# --------------------------------------------------------------------------
CASES = [
    # b, s, h, dk, dv, beta_max, gated, random_state, channel
    (2, 16, 3, 8, 8, 0.95, False, False, False),
    (2, 16, 3, 8, 8, 0.95, True, False, False),
    (2, 12, 2, 8, 16, 0.95, True, True, False),
    (2, 12, 2, 8, 8, 1.95, True, True, False),
    (2, 13, 2, 8, 8, 0.95, True, True, False),
    (1, 5, 1, 4, 4, 0.95, False, False, False),
    (2, 16, 3, 8, 8, 0.95, True, False, True),
    (2, 40, 2, 8, 8, 0.95, True, True, True),
    (1, 37, 1, 4, 6, 1.95, True, True, True),
    (2, 16, 2, 16, 8, 0.95, True, True, True),
    (2, 100, 2, 64, 64, 0.95, True, True, False),
    (1, 70, 2, 128, 128, 0.95, True, True, True),
    (1, 33, 1, 256, 40, 0.95, True, True, True),
    (1, 45, 2, 96, 72, 1.5, True, True, False),
]


@pytest.mark.parametrize("b,s,h,dk,dv,beta_max,gated,rs,channel", CASES)
def test_chunk_matches_the_oracle_fp32(b, s, h, dk, dv, beta_max, gated, rs, channel):
    raw = random_raw(np.random.default_rng(100 + s + dk), b, s, h, dk, dv, beta_max, gated, rs, channel)
    y0, s0 = oracle_run(raw)
    y, st = gpu_chunk(raw)
    assert rel_err(y, y0) < F32_TOL
    assert rel_err(st, s0) < F32_TOL


@pytest.mark.parametrize("b,s,h,dk,dv,beta_max,gated,rs,channel", CASES)
def test_step_matches_the_oracle_fp32(b, s, h, dk, dv, beta_max, gated, rs, channel):
    """The fused decode tick, run over the sequence (DeltaPath::Recurrent)."""
    raw = random_raw(np.random.default_rng(200 + s + dk), b, s, h, dk, dv, beta_max, gated, rs, channel)
    y0, s0 = oracle_run(raw)
    inp = dn.DeltaInput(*(to_dev(raw[n]) for n in ("q", "k", "v", "erase", "write", "g", "state")))
    y, st = inp.run(dn.DeltaPath.Recurrent())
    assert rel_err(y, y0) < F32_TOL
    assert rel_err(st, s0) < F32_TOL


@pytest.mark.parametrize("beta,gated", [(0.9, False), (0.9, True), (1.8, True)])
def test_chunk_on_a_constant_input(beta, gated):
    """src/delta/tests.rs:423-460: the WY conditioning known-answer test."""
    raw = constant_raw(np.random.default_rng(7), 2, 128, 2, 8, 8, beta, gated)
    y0, s0 = oracle_run(raw)
    y, st = gpu_chunk(raw)
    assert rel_err(y, y0) < F32_TOL and rel_err(st, s0) < F32_TOL


def test_split_calls_match_a_single_call():
    """src/delta/tests.rs:465-494, including the in-place state update."""
    raw = random_raw(np.random.default_rng(8), 2, 150, 2, 32, 32, 0.95, True, False)
    dev = {n: to_dev(raw[n]) for n in ("q", "k", "v", "erase", "write", "g", "state")}
    sc = 1 / np.sqrt(32)
    y_all, s_all = dn.delta_chunk_recalculated(*(dev[n] for n in ("q", "k", "v", "erase", "write", "g", "state")),
                                               True, 64, sc)
    st = dev["state"].clone()
    parts = []
    for a, n in ((0, 7), (7, 64), (71, 79)):
        cut = {k: dev[k][:, a:a + n].contiguous() for k in ("q", "k", "v", "erase", "write", "g")}
        y, _ = dn.delta_chunk_recalculated(cut["q"], cut["k"], cut["v"], cut["erase"], cut["write"], cut["g"],
                                           st, True, 64, sc, state_out=st)
        parts.append(y)
    torch.cuda.synchronize()
    assert (torch.cat(parts, 1) - y_all).abs().max().item() < 1e-5
    assert (st - s_all).abs().max().item() < 1e-5


def test_a_zero_gate_is_the_ungated_delta_rule():
    raw = random_raw(np.random.default_rng(9), 2, 40, 2, 16, 16, 0.95, False, True)
    y0, s0 = gpu_chunk(raw)
    y1, s1 = gpu_chunk(dict(raw, g=np.zeros(raw["erase"].shape)))
    assert (y0 - y1).abs().max().item() < 1e-6 and (s0 - s1).abs().max().item() < 1e-6


def test_broadcast_channel_gates_are_the_scalar_delta_rule():
    raw = random_raw(np.random.default_rng(10), 2, 50, 2, 16, 24, 0.95, True, True)
    wide = dict(raw, erase=np.repeat(raw["erase"], 16, 3), write=np.repeat(raw["write"], 24, 3),
                g=np.repeat(raw["g"], 16, 3))
    y0, s0 = gpu_chunk(raw)
    y1, s1 = gpu_chunk(wide)
    assert rel_err(y0, y1.double().cpu().numpy()) < 1e-5 and rel_err(s0, s1.double().cpu().numpy()) < 1e-5


# --------------------------------------------------------------------------
# Micro-steps in-kernel (DeltaProduct / GDN-2 fold).
# --------------------------------------------------------------------------
@pytest.mark.parametrize("u", [1, 2, 3])
@pytest.mark.parametrize("cfg", [4, 5])
def test_householder_fold_in_kernel(u, cfg):
    raw = config_inputs(cfg, np.random.default_rng(11 + u), 2, 45, 2, 32, 32, u=u)
    if cfg == 5:  # keep the per-channel decay mild enough for a long readout
        raw["g"] = raw["g"] * 0.05
    y0, s0 = oracle_run(raw, u)
    y, st = gpu_chunk(raw, u=u)
    assert rel_err(y, y0) < F32_TOL and rel_err(st, s0) < F32_TOL
    # the step kernel's fold: token by token
    inp = dn.DeltaInput(*(to_dev(raw[n]) for n in ("q", "k", "v", "erase", "write", "g", "state")),
                        n_householder=u)
    y2, s2 = inp.run(dn.DeltaPath.Recurrent())
    assert rel_err(y2, y0) < F32_TOL and rel_err(s2, s0) < F32_TOL


# --------------------------------------------------------------------------
# bf16 inputs, fp32 state and accumulation.
# --------------------------------------------------------------------------
@pytest.mark.parametrize("cfg", [1, 2, 4, 5])
def test_bf16_inputs_simt(cfg):
    u = 2 if cfg == 4 else 1
    raw = config_inputs(cfg, np.random.default_rng(12), 1, 96, 2, 64, 64, u=u)
    y0, s0 = oracle_run(raw, u, in_dtype=torch.bfloat16, gate_dtype=torch.bfloat16)
    y, st = gpu_chunk(raw, u=u, in_dtype=torch.bfloat16, gate_dtype=torch.bfloat16, force_simt=True)
    assert rel_err(y, y0) < F32_TOL and rel_err(st, s0) < F32_TOL


def test_decode_1024_steps_state_parity():
    """BASELINE config 3's decode at reduced batch: 1024 fused ticks from a
    N(0, 0.02^2) state, bf16 q/k/v, fp32 state; final state within 1e-4
    relative of the float64 oracle on the same rounded inputs."""
    rng = np.random.default_rng(13)
    b, h, d, steps = 2, 4, 128, 1024
    raw = config_inputs(3, rng, b, steps, h, d, d)
    raw["state"] = rng.normal(0.0, 0.02, (b, h, d, d))
    y0, s0 = oracle_run(raw, 1, in_dtype=torch.bfloat16)
    dev = {n: to_dev(raw[n], torch.bfloat16 if n in ("q", "k", "v") else torch.float32)
           for n in ("q", "k", "v", "erase", "write", "g")}
    st = to_dev(raw["state"])
    ys = []
    sc = 1 / np.sqrt(d)
    for t in range(steps):
        y, _ = dn.delta_step(*(dev[n][:, t].contiguous() for n in ("q", "k", "v", "erase", "write", "g")), st, sc,
                             out_dtype=torch.float32, state_out=st)
        ys.append(y)
    torch.cuda.synchronize()
    assert rel_err(st, s0) < F32_TOL
    assert rel_err(torch.stack(ys, 1), y0) < F32_TOL


def test_step_in_place_and_out_of_place_agree():
    rng = np.random.default_rng(14)
    raw = config_inputs(5, rng, 3, 1, 2, 128, 128)
    raw["state"] = rng.normal(0, 0.2, (3, 2, 128, 128))
    dev = {n: to_dev(raw[n])[:, 0].contiguous() for n in ("q", "k", "v", "erase", "write", "g")}
    st = to_dev(raw["state"])
    y0, s0 = dn.delta_step(dev["q"], dev["k"], dev["v"], dev["erase"], dev["write"], dev["g"], st, 0.1)
    st2 = st.clone()
    y1, _ = dn.delta_step(dev["q"], dev["k"], dev["v"], dev["erase"], dev["write"], dev["g"], st2, 0.1,
                          state_out=st2)
    torch.cuda.synchronize()
    assert torch.equal(y0, y1) and torch.equal(s0, st2)


@pytest.mark.parametrize("widths,in_dtype,out_dtype", [
    ((1, 1, 1), torch.bfloat16, torch.float32),
    ((128, 128, 128), torch.bfloat16, torch.bfloat16),
    ((1, 128, 0), torch.float32, torch.float32),
    ((128, 1, 1), torch.float32, torch.bfloat16),
])
def test_step_stream_matches_the_per_tile_kernel(widths, in_dtype, out_dtype):
    """The streaming decode kernel (one CTA per SM walking 1024 heads through a three-slot ring; it serves
    ticks of at least 1024 heads) against the per-tile kernel, in place and out of place."""
    ew, ww, gw = widths
    rng = np.random.default_rng(15 + ew + gw)
    b, h, d = 256, 4, 128
    raw = config_inputs(5, rng, b, 1, h, d, d)
    raw["erase"], raw["write"] = raw["erase"][..., :ew], raw["write"][..., :ww]
    raw["g"] = None if gw == 0 else raw["g"][..., :gw]
    st = to_dev(rng.normal(0, 0.05, (b, h, d, d)))
    dev = {n: None if raw[n] is None else to_dev(raw[n], in_dtype if n in ("q", "k", "v") else torch.float32)[:, 0]
           .contiguous() for n in ("q", "k", "v", "erase", "write", "g")}
    args = (dev["q"], dev["k"], dev["v"], dev["erase"], dev["write"], dev["g"])
    y0, s0 = dn.delta_step(*args, st, 0.09, out_dtype=out_dtype, force_simt=True)
    y1, s1 = dn.delta_step(*args, st, 0.09, out_dtype=out_dtype)
    st2 = st.clone()
    y2, _ = dn.delta_step(*args, st2, 0.09, out_dtype=out_dtype, state_out=st2)
    torch.cuda.synchronize()
    tol = 1e-2 if out_dtype == torch.bfloat16 else 1e-5
    assert (y0.float() - y1.float()).abs().max().item() < tol
    assert (s0 - s1).abs().max().item() < 1e-5
    assert torch.equal(y1, y2) and torch.equal(s1, st2)
    assert abi.lib().dc_device_status(1) == 0


def test_step_stream_repeat_calls_are_bit_identical():
    """The streaming decode kernel's producer and consumers share a three-slot ring: repeated ticks from the
    same state, and a subset of the heads, must agree bit for bit."""
    rng = np.random.default_rng(51)
    b, h, d = 300, 4, 128  # 1200 heads: every CTA walks several heads through the ring
    raw = config_inputs(5, rng, b, 1, h, d, d)
    st = to_dev(rng.normal(0, 0.05, (b, h, d, d)))
    dv = {n: to_dev(raw[n], torch.bfloat16 if n in ("q", "k", "v") else torch.float32)[:, 0].contiguous()
          for n in ("q", "k", "v", "erase", "write", "g")}
    args = (dv["q"], dv["k"], dv["v"], dv["erase"], dv["write"], dv["g"])
    y0, s0 = dn.delta_step(*args, st, 0.09, out_dtype=torch.float32)
    for _ in range(4):
        y, s = dn.delta_step(*args, st, 0.09, out_dtype=torch.float32)
        assert torch.equal(y, y0) and torch.equal(s, s0)
    sub = slice(7, 263)  # 1024 heads: still the streaming kernel (it serves ticks of at least 1024 heads)
    y, s = dn.delta_step(*(t[sub].contiguous() for t in args), st[sub].contiguous(), 0.09, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(y, y0[sub]) and torch.equal(s, s0[sub])
    assert abi.lib().dc_device_status(1) == 0

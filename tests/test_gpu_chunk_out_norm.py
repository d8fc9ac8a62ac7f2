"""GPU parity of the prefill with the output norm after it (dc_chunk_fwd_out_norm).

A layer's forward normalises the core's read-out over each head's dv values before out_proj
(OutNorm, src/common/norm.rs:106-144, on the y of chunk_recalculated.rs:115-126).  The plain norm is
applied inside the fused tensor-core prefill's read-out, from its float32 accumulator; a gated norm, or a
prefill served by another kernel, runs the prefill and then dc_out_norm in place on y.

Checks, on ragged sequences (T = 200: the last chunk is partial) at d = 128:
* against the float64 oracle: the recurrence (oracle.householder) followed by oracle.out_norm, within
  the north star's 2e-2 for bf16 q/k/v (values are O(weight) after the norm);
* against the same library's two calls (prefill with float32 y, then dc_out_norm): 1e-5 for float32 y,
  one bf16 ulp (2^-7 relative) for bf16 y; the final state bit-identical to the plain prefill's;
* which path ran, from dc_chunk_fwd_out_norm_fused."""
import importlib
import math

import numpy as np
import pytest
import torch

import oracle
from _inputs import config_inputs

pytestmark = pytest.mark.gpu
dn = importlib.import_module("burn-deltanet_b200")
abi = importlib.import_module("burn-deltanet_b200._abi")

TOL = 2e-2
D = 128


def _inputs(kind, u, seed, b=2, t=200, h=3):
    rng = np.random.default_rng(seed)
    raw = config_inputs(kind, rng, b, t, h, D, D, u=u)
    raw["state"] = rng.normal(0, 0.05, (b, h, D, D))
    dev = {}
    for n in ("q", "k", "v", "erase", "write", "g", "state"):
        if raw[n] is None:
            dev[n] = None
            continue
        x = torch.from_numpy(np.ascontiguousarray(raw[n])).to("cuda", torch.float32)
        dev[n] = x.to(torch.bfloat16) if n in ("q", "k", "v") else x
    # the oracle sees exactly what the kernels see: q, k, v rounded to bf16
    for n in ("q", "k", "v"):
        raw[n] = dev[n].double().cpu().numpy()
    w = torch.from_numpy(rng.uniform(0.5, 1.5, D)).to("cuda", torch.float32)
    return raw, dev, w


def _args(dev, u):
    gated = dev["g"] is not None
    return (dev["q"], dev["k"], dev["v"], dev["erase"], dev["write"], dev["g"], dev["state"], gated, 64,
            1.0 / math.sqrt(D))


@pytest.mark.parametrize("kind,u,out_dtype,norm_gated,fused", [
    ("gdn", 1, torch.bfloat16, False, True),
    ("gdn", 1, torch.float32, False, True),
    ("deltanet", 1, torch.float32, False, True),
    ("deltaproduct", 2, torch.bfloat16, False, True),
    ("deltaproduct", 3, torch.float32, False, True),
    ("gdn", 1, torch.bfloat16, True, False),   # gated norm: the two kernels
    ("gdn2", 1, torch.float32, False, False),  # per-channel gates: the split prefill, then the norm
])
def test_chunk_out_norm_matches_the_oracle(kind, u, out_dtype, norm_gated, fused):
    raw, dev, w = _inputs(kind, u, seed=7 + u + (3 if norm_gated else 0))
    args = _args(dev, u)
    b, t, h = dev["q"].shape[:3]
    gate = None
    if norm_gated:
        gate = (torch.randn(b, t, h, D, device="cuda", generator=torch.Generator("cuda").manual_seed(5)) * 2)
        gate = gate.to(out_dtype)
    eps = 1e-5
    assert dn.chunk_out_norm_is_fused(*args[:9], w, gate, n_householder=u, out_dtype=out_dtype) is fused
    assert abi.lib().dc_device_status(1) == 0
    y, s = dn.delta_chunk_recalculated_out_norm(*args, w, gate, eps, n_householder=u, out_dtype=out_dtype)
    # the same library's two calls, through a float32 read-out
    y32, s32 = dn.delta_chunk_recalculated(*args, n_householder=u, out_dtype=torch.float32)
    y2 = dn.out_norm(y32, None if gate is None else gate.float(), w, eps, out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert abi.lib().dc_device_status(1) == 0
    assert y.dtype == out_dtype and tuple(y.shape) == (b, t, h, D)
    assert torch.isfinite(y).all()
    assert torch.equal(s, s32), "the norm must leave the final state alone"

    y_o, _ = oracle.householder("recurrent", raw["q"], raw["k"], raw["v"], raw["erase"], raw["write"], raw["g"],
                                raw["state"], u, scale=1.0 / math.sqrt(D))
    ref = oracle.out_norm(y_o, None if gate is None else gate.double().cpu().numpy(), w.double().cpu().numpy(), eps)
    got = y.double().cpu().numpy()
    e_oracle = np.abs(got - ref).max() / max(1.0, np.abs(ref).max())
    e_two = ((y.double() - y2.double()).abs() / y2.double().abs().clamp_min(1.0)).max().item()
    print(f"{kind} u={u} {out_dtype} gated={norm_gated}: vs oracle {e_oracle:.2e}, vs two calls {e_two:.2e}")
    assert e_oracle < TOL, e_oracle
    if out_dtype == torch.float32:
        assert e_two < 1e-5, e_two
    elif gate is not None:
        # the two-kernel path rounds y to bf16 before the norm (the second call here reads float32), then
        # rounds the result: two bf16 roundings
        assert e_two <= 2 ** -6, e_two
    else:
        assert e_two <= 2 ** -7, e_two  # one bf16 ulp: the same float32 values rounded once


def test_chunk_out_norm_two_kernel_path_is_prefill_then_norm_bit_for_bit():
    """Where the norm is not fused, the call is dc_chunk_fwd then dc_out_norm in place on y: the results
    equal those two public calls exactly."""
    raw, dev, w = _inputs("gdn", 1, seed=21)
    args = _args(dev, 1)
    gate = torch.randn(dev["q"].shape[:3] + (D,), device="cuda").to(torch.bfloat16)
    y, s = dn.delta_chunk_recalculated_out_norm(*args, w, gate, 1e-6, out_dtype=torch.bfloat16)
    y0, s0 = dn.delta_chunk_recalculated(*args, out_dtype=torch.bfloat16)
    y1 = dn.out_norm(y0, gate, w, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(y, y1) and torch.equal(s, s0)


def test_chunk_out_norm_repeat_calls_are_bit_identical_and_rows_of_zeros_stay_zero():
    """Two fused calls agree bit for bit; with v = 0 and S0 = 0 every read-out row is zero and the norm
    returns zeros (the eps guard), not NaN."""
    raw, dev, w = _inputs("gdn", 1, seed=33)
    args = _args(dev, 1)
    y1, s1 = dn.delta_chunk_recalculated_out_norm(*args, w, out_dtype=torch.bfloat16)
    y2, s2 = dn.delta_chunk_recalculated_out_norm(*args, w, out_dtype=torch.bfloat16)
    zv = torch.zeros_like(dev["v"])
    zs = torch.zeros_like(dev["state"])
    zargs = args[:2] + (zv,) + args[3:6] + (zs,) + args[7:]
    yz, sz = dn.delta_chunk_recalculated_out_norm(*zargs, w, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2) and torch.equal(s1, s2)
    assert torch.equal(yz, torch.zeros_like(yz)) and torch.equal(sz, zs)
    assert abi.lib().dc_device_status(1) == 0


def test_chunk_out_norm_on_the_fp32_chunked_path():
    """float32 q / k / v take the fp32-accurate chunked prefill; the plain norm then runs as dc_out_norm in
    place on y, within the fp32 path's 1e-4 of the float64 recurrence and norm."""
    rng = np.random.default_rng(41)
    raw = config_inputs("gdn", rng, 2, 150, 3, 64, 64)
    raw["state"] = rng.normal(0, 0.05, (2, 3, 64, 64))
    dev = {n: None if raw[n] is None else torch.from_numpy(np.ascontiguousarray(raw[n])).to("cuda", torch.float32)
           for n in ("q", "k", "v", "erase", "write", "g", "state")}
    w = torch.from_numpy(rng.uniform(0.5, 1.5, 64)).to("cuda", torch.float32)
    args = (dev["q"], dev["k"], dev["v"], dev["erase"], dev["write"], dev["g"], dev["state"], True, 64,
            1.0 / math.sqrt(64))
    assert dn.chunk_out_norm_is_fused(*args[:9], w) is False
    y, s = dn.delta_chunk_recalculated_out_norm(*args, w, None, 1e-5)
    torch.cuda.synchronize()
    y_o, s_o = oracle.householder("recurrent", raw["q"], raw["k"], raw["v"], raw["erase"], raw["write"], raw["g"],
                                  raw["state"], 1, scale=1.0 / math.sqrt(64))
    ref = oracle.out_norm(y_o, None, w.double().cpu().numpy(), 1e-5)
    e_y = np.abs(y.double().cpu().numpy() - ref).max() / max(1.0, np.abs(ref).max())
    e_s = np.abs(s.double().cpu().numpy() - s_o).max() / max(1.0, np.abs(s_o).max())
    assert e_y < 1e-4 and e_s < 1e-4, (e_y, e_s)
    assert abi.lib().dc_device_status(1) == 0

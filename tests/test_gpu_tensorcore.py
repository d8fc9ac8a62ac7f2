"""GPU parity of the tensor-core (tcgen05) chunk kernel: bf16 q/k/v, fp32
gates, fp32 state and accumulation, dk = dv = 128.

Bar: max |gpu - oracle| < 2e-2 on y and on the final state, the oracle
(float64) run on the same bf16-rounded inputs; and the kernel's device
status word stays 0 (no bounded wait ran out)."""
import importlib

import numpy as np
import pytest
import torch

import oracle
from _inputs import config_inputs, constant_raw, random_raw

pytestmark = pytest.mark.gpu
dn = importlib.import_module("burn-deltanet_b200")
abi = importlib.import_module("burn-deltanet_b200._abi")

BF16_TOL = 2e-2


def dev(x, dtype=torch.float32):
    return None if x is None else torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


def run_tc(raw, force_simt=False, out_dtype=torch.float32):
    q, k, v = (dev(raw[n], torch.bfloat16) for n in ("q", "k", "v"))
    e, w, g = (dev(raw[n]) for n in ("erase", "write", "g"))
    st = dev(raw["state"])
    y, s = dn.delta_chunk_recalculated(q, k, v, e, w, g, st, g is not None, 64, 1 / np.sqrt(128),
                                       out_dtype=out_dtype, force_simt=force_simt)
    torch.cuda.synchronize()
    return y.double().cpu().numpy(), s.double().cpu().numpy(), (q, k, v)


def reference(raw, qkv):
    q, k, v = (t.double().cpu().numpy() for t in qkv)
    return oracle.recurrent(q, k, v, raw["erase"], raw["write"], raw["g"], raw["state"])


def kernel_choice(raw):
    a = abi.ChunkArgs()
    b, s, h, d = raw["q"].shape
    a.batch, a.seq, a.heads, a.dk, a.dv = b, s, h, d, raw["v"].shape[3]
    a.n_householder, a.erase_w, a.write_w = 1, raw["erase"].shape[3], raw["write"].shape[3]
    a.g_w = 0 if raw["g"] is None else raw["g"].shape[3]
    a.chunk_len, a.in_dtype, a.gate_dtype, a.out_dtype, a.scale = 64, abi.DC_BF16, abi.DC_F32, abi.DC_F32, 0.1
    a.q = a.k = a.v = a.erase = a.write = a.g = 1 << 20
    a.state_in = a.state_out = 2 << 20
    a.y = 3 << 20
    return abi.lib().dc_chunk_kernel_choice(a)


def check(raw, tol=BF16_TOL):
    assert kernel_choice(raw) == 1, "expected the tensor-core kernel"
    assert abi.lib().dc_device_status(1) == 0
    y, s, qkv = run_tc(raw)
    assert abi.lib().dc_device_status(1) == 0, "a bounded wait in the kernel ran out"
    y0, s0 = reference(raw, qkv)
    ey, es = np.abs(y - y0).max(), np.abs(s - s0).max()
    print(f"max |y - ref| {ey:.3e} (|ref| {np.abs(y0).max():.2f}); max |S - ref| {es:.3e} (|ref| {np.abs(s0).max():.2f})")
    assert ey < tol and es < tol, (ey, es)
    return ey, es


@pytest.mark.parametrize("seq", [64, 1, 63, 65, 200, 1000])
def test_deltanet_prefill(seq):
    check(config_inputs(2, np.random.default_rng(seq), 2, seq, 3, 128, 128))


def test_deltanet_negative_eigenvalues():
    check(config_inputs(2, np.random.default_rng(5), 2, 300, 2, 128, 128, neg_eig=True))


@pytest.mark.parametrize("seq", [64, 130, 777])
def test_gated_deltanet_prefill(seq):
    check(config_inputs(1, np.random.default_rng(seq + 7), 2, seq, 2, 128, 128))


def test_carried_state_and_reference_gates():
    raw = random_raw(np.random.default_rng(3), 2, 150, 2, 128, 128, 0.95, True, True)
    check(raw)


def test_constant_input():
    check(constant_raw(np.random.default_rng(4), 1, 256, 2, 128, 128, 1.8, True))


def test_long_sequence_drift():
    """bf16 operands against the fp32 state over 4096 steps (the config 2 length)."""
    ey, es = check(config_inputs(2, np.random.default_rng(6), 1, 4096, 2, 128, 128))
    print(f"T=4096 max err y {ey:.3e} state {es:.3e}")


def test_matches_the_cuda_core_kernel():
    raw = config_inputs(1, np.random.default_rng(8), 2, 333, 4, 128, 128)
    y1, s1, _ = run_tc(raw)
    y2, s2, _ = run_tc(raw, force_simt=True)
    assert np.abs(y1 - y2).max() < BF16_TOL and np.abs(s1 - s2).max() < BF16_TOL


def test_bf16_output():
    raw = config_inputs(2, np.random.default_rng(9), 1, 128, 2, 128, 128)
    y, s, qkv = run_tc(raw, out_dtype=torch.bfloat16)
    y0, s0 = reference(raw, qkv)
    assert np.abs(y - y0).max() < BF16_TOL and np.abs(s - s0).max() < BF16_TOL


# ---------------------------------------------------------------------------
# DeltaProduct: u micro-steps folded inside the tensor-core kernel
# (src/delta_product/delta_product.rs:178-228), config 4's recipe.
# ---------------------------------------------------------------------------
def run_tc_fold(raw, u):
    q, k, v = (dev(raw[n], torch.bfloat16) for n in ("q", "k", "v"))
    e, w, g = (dev(raw[n]) for n in ("erase", "write", "g"))
    st = dev(raw["state"])
    y, s = dn.delta_chunk_recalculated(q, k, v, e, w, g, st, g is not None, 64, 1 / np.sqrt(128),
                                       n_householder=u, out_dtype=torch.float32)
    torch.cuda.synchronize()
    rq, rk, rv = (t.double().cpu().numpy() for t in (q, k, v))
    y0, s0 = oracle.householder("recurrent", rq, rk, rv, raw["erase"], raw["write"], raw["g"], raw["state"], u)
    return y.double().cpu().numpy(), s.double().cpu().numpy(), y0, s0


@pytest.mark.parametrize("u,seq", [(2, 64), (2, 97), (3, 64), (3, 130), (4, 50)])
def test_deltaproduct_fold(u, seq):
    raw = config_inputs(4, np.random.default_rng(20 + u + seq), 2, seq, 2, 128, 128, u=u)
    a = abi.ChunkArgs()
    a.batch, a.seq, a.heads, a.dk, a.dv, a.n_householder = 2, seq, 2, 128, 128, u
    a.erase_w = a.write_w = a.g_w = 1
    a.chunk_len, a.in_dtype, a.gate_dtype, a.out_dtype, a.scale = 64, abi.DC_BF16, abi.DC_F32, abi.DC_F32, 0.1
    a.q = a.k = a.v = a.erase = a.write = a.g = 1 << 20
    a.state_in = a.state_out = 2 << 20
    a.y = 3 << 20
    assert abi.lib().dc_chunk_kernel_choice(a) == 1
    assert abi.lib().dc_device_status(1) == 0
    y, s, y0, s0 = run_tc_fold(raw, u)
    assert abi.lib().dc_device_status(1) == 0
    ey, es = np.abs(y - y0).max(), np.abs(s - s0).max()
    print(f"u={u} T={seq}: max |y - ref| {ey:.3e}; max |S - ref| {es:.3e} (|ref| {np.abs(s0).max():.2f})")
    assert ey < BF16_TOL and es < BF16_TOL


def test_deltaproduct_fold_ungated():
    raw = config_inputs(4, np.random.default_rng(31), 1, 150, 3, 128, 128, u=2)
    raw["g"] = None
    y, s, y0, s0 = run_tc_fold(raw, 2)
    assert np.abs(y - y0).max() < BF16_TOL and np.abs(s - s0).max() < BF16_TOL


@pytest.mark.parametrize("cfg,u,out_dtype", [(3, 1, torch.float32), (4, 2, torch.float32), (4, 3, torch.bfloat16),
                                             (3, 1, torch.bfloat16)])
def test_repeat_calls_are_bit_identical(cfg, u, out_dtype):
    """The kernel's roles hand buffers to each other through mbarriers only; a buffer reused too early shows
    up as run-to-run differences.  Gated inputs (the gate slots are read by both roles), several chunks,
    five calls, and a one-sequence call against its rows of the batched one."""
    raw = config_inputs(cfg, np.random.default_rng(31 + u), 3, 200, 2, 128, 128, u=u)
    raw["state"] = np.random.default_rng(32).normal(0, 0.02, raw["state"].shape)
    q, k, v = (dev(raw[n], torch.bfloat16) for n in ("q", "k", "v"))
    e, w, g, st = (dev(raw[n]) for n in ("erase", "write", "g", "state"))

    def call(sl=slice(None)):
        y, s = dn.delta_chunk_recalculated(q[sl].contiguous(), k[sl].contiguous(), v[sl].contiguous(),
                                           e[sl].contiguous(), w[sl].contiguous(), g[sl].contiguous(),
                                           st[sl].contiguous(), True, 64, 1 / np.sqrt(128), n_householder=u,
                                           out_dtype=out_dtype)
        torch.cuda.synchronize()
        return y, s

    assert abi.lib().dc_chunk_kernel_choice is not None
    y0, s0 = call()
    for _ in range(4):
        y, s = call()
        assert torch.equal(y, y0) and torch.equal(s, s0)
    for b in range(3):
        y, s = call(slice(b, b + 1))
        assert torch.equal(y, y0[b:b + 1]) and torch.equal(s, s0[b:b + 1])
    assert abi.lib().dc_device_status(1) == 0

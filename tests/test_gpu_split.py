"""GPU parity of the two-kernel tensor-core path (per-channel gates, GDN-2):
the chunk-parallel prep kernel and the state-scan kernel over a workspace.

Bar: max |gpu - oracle| < 2e-2 on y and on the final state, the oracle
(float64 recurrence, the exact definition) run on the same bf16-rounded
inputs; the device status word stays 0 (no bounded wait ran out).  Config 5
is checked against the recurrence because the reference chunk path clamps
its decay exponents for gates that strong."""
import importlib

import numpy as np
import pytest
import torch

import oracle
from _inputs import config_inputs

pytestmark = pytest.mark.gpu
dn = importlib.import_module("burn-deltanet_b200")
abi = importlib.import_module("burn-deltanet_b200._abi")

BF16_TOL = 2e-2


def dev(x, dtype=torch.float32):
    return None if x is None else torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


def args_of(raw, flags=0, workspace=0, workspace_bytes=0):
    a = abi.ChunkArgs()
    b, s, h, d = raw["q"].shape
    a.batch, a.seq, a.heads, a.dk, a.dv = b, s, h, d, raw["v"].shape[3]
    a.n_householder, a.erase_w, a.write_w = 1, raw["erase"].shape[3], raw["write"].shape[3]
    a.g_w = 0 if raw["g"] is None else raw["g"].shape[3]
    a.chunk_len, a.in_dtype, a.gate_dtype, a.out_dtype, a.scale = 64, abi.DC_BF16, abi.DC_F32, abi.DC_F32, 0.1
    a.q = a.k = a.v = a.erase = a.write = a.g = 1 << 20
    a.state_in = a.state_out = 2 << 20
    a.y = 3 << 20
    a.flags = flags
    a.workspace, a.workspace_bytes = workspace, workspace_bytes
    return a


def run_split(raw, force_split=False, out_dtype=torch.float32, workspace=None):
    q, k, v = (dev(raw[n], torch.bfloat16) for n in ("q", "k", "v"))
    e, w, g = (dev(raw[n]) for n in ("erase", "write", "g"))
    st = dev(raw["state"])
    y, s = dn.delta_chunk_recalculated(q, k, v, e, w, g, st, g is not None, 64, 1 / np.sqrt(128),
                                       out_dtype=out_dtype, force_split=force_split, workspace=workspace)
    torch.cuda.synchronize()
    return y.double().cpu().numpy(), s.double().cpu().numpy(), (q, k, v)


def reference(raw, qkv):
    q, k, v = (t.double().cpu().numpy() for t in qkv)
    return oracle.recurrent(q, k, v, raw["erase"], raw["write"], raw["g"], raw["state"])


def check(raw, force_split=False, out_dtype=torch.float32, tol=BF16_TOL):
    flags = abi.DC_FLAG_FORCE_SPLIT if force_split else 0
    a = args_of(raw, flags)
    need = abi.lib().dc_chunk_workspace_size(a)
    assert need > 0, "expected the two-kernel path to apply"
    a.workspace, a.workspace_bytes = 4 << 20, need
    assert abi.lib().dc_chunk_kernel_choice(a) == 2
    assert abi.lib().dc_chunk_launches(a) == 2
    assert abi.lib().dc_device_status(1) == 0
    y, s, qkv = run_split(raw, force_split, out_dtype)
    assert abi.lib().dc_device_status(1) == 0, "a bounded wait in the kernels ran out"
    y0, s0 = reference(raw, qkv)
    ey, es = np.abs(y - y0).max(), np.abs(s - s0).max()
    print(f"max |y - ref| {ey:.3e} (|ref| {np.abs(y0).max():.2f}); max |S - ref| {es:.3e} (|ref| {np.abs(s0).max():.2f})")
    assert np.isfinite(y).all() and np.isfinite(s).all()
    assert ey < tol and es < tol, (ey, es)
    return ey, es


@pytest.mark.parametrize("seq", [64, 1, 63, 65, 200, 1000])
def test_gdn2_prefill(seq):
    check(config_inputs(5, np.random.default_rng(seq), 2, seq, 2, 128, 128))


def test_gdn2_carried_state():
    raw = config_inputs(5, np.random.default_rng(11), 2, 300, 2, 128, 128)
    raw["state"] = np.random.default_rng(12).normal(0, 0.02, raw["state"].shape)
    check(raw)


def test_gdn2_long_sequence():
    """Config-5 gates over 64 chunks: the decay factors underflow freely and the state stays on track."""
    check(config_inputs(5, np.random.default_rng(13), 1, 4096, 2, 128, 128))


@pytest.mark.parametrize("widths", [(128, 1, 128), (1, 128, 128), (128, 128, 1), (1, 1, 128), (128, 128, 0),
                                    (128, 1, 0)])
def test_gate_width_mixes(widths):
    """Every broadcast combination that has a per-channel gate somewhere."""
    ew, ww, gw = widths
    raw = config_inputs(5, np.random.default_rng(sum(widths)), 2, 150, 2, 128, 128)
    raw["erase"] = raw["erase"][..., :ew].copy()
    raw["write"] = raw["write"][..., :ww].copy()
    raw["g"] = None if gw == 0 else raw["g"][..., :gw].copy()
    check(raw)


@pytest.mark.parametrize("cfg,seq", [(2, 200), (1, 333)])
def test_forced_split_per_head(cfg, seq):
    check(config_inputs(cfg, np.random.default_rng(cfg * seq), 2, seq, 3, 128, 128), force_split=True)


def test_forced_split_negative_eigenvalues():
    check(config_inputs(2, np.random.default_rng(5), 2, 300, 2, 128, 128, neg_eig=True), force_split=True)


def test_bf16_output():
    """bf16 y leaves through the TMA store; compared at bf16 resolution."""
    check(config_inputs(5, np.random.default_rng(21), 2, 257, 2, 128, 128), out_dtype=torch.bfloat16,
          tol=BF16_TOL + 1e-2)


def test_split_matches_fused():
    """The same per-head problem through both tensor-core paths."""
    raw = config_inputs(1, np.random.default_rng(31), 2, 500, 2, 128, 128)
    ys, ss, _ = run_split(raw, force_split=True)
    q, k, v = (dev(raw[n], torch.bfloat16) for n in ("q", "k", "v"))
    e, w, g = (dev(raw[n]) for n in ("erase", "write", "g"))
    yf, sf = dn.delta_chunk_recalculated(q, k, v, e, w, g, dev(raw["state"]), True, 64, 1 / np.sqrt(128),
                                         out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert np.abs(ys - yf.double().cpu().numpy()).max() < BF16_TOL
    assert np.abs(ss - sf.double().cpu().numpy()).max() < BF16_TOL


def test_workspace_reuse_and_errors():
    raw = config_inputs(5, np.random.default_rng(41), 1, 130, 2, 128, 128)
    a = args_of(raw)
    need = abi.lib().dc_chunk_workspace_size(a)
    # no workspace: the CUDA-core kernel serves the call
    assert abi.lib().dc_chunk_kernel_choice(a) == 0
    # a workspace that is too small is an error, not a silent fallback
    a.workspace, a.workspace_bytes = 4 << 20, need - 1
    assert abi.lib().dc_chunk_kernel_choice(a) == -abi.DC_EWORKSPACE
    ws = torch.empty(need - 16, dtype=torch.uint8, device="cuda")
    with pytest.raises(dn.DeltaCoreError) as err:
        run_split(raw, workspace=ws)
    assert err.value.status == abi.DC_EWORKSPACE
    # one workspace serves two calls in a row
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    y1, s1, qkv = run_split(raw, workspace=ws)
    y2, s2, _ = run_split(raw, workspace=ws)
    assert np.array_equal(y1, y2) and np.array_equal(s1, s2)
    y0, s0 = reference(raw, qkv)
    assert np.abs(y1 - y0).max() < BF16_TOL and np.abs(s1 - s0).max() < BF16_TOL


def test_repeat_calls_are_bit_identical():
    """Prep and scan hand the workspace over between kernels and the scan's roles meet on mbarriers: run-to-run
    and batched-vs-single-sequence results must agree bit for bit."""
    raw = config_inputs(5, np.random.default_rng(41), 3, 330, 2, 128, 128)
    raw["state"] = np.random.default_rng(42).normal(0, 0.02, raw["state"].shape)
    q, k, v = (dev(raw[n], torch.bfloat16) for n in ("q", "k", "v"))
    e, w, g, st = (dev(raw[n]) for n in ("erase", "write", "g", "state"))

    def call(sl=slice(None)):
        y, s = dn.delta_chunk_recalculated(*(t[sl].contiguous() for t in (q, k, v, e, w, g, st)), True, 64,
                                           1 / np.sqrt(128), out_dtype=torch.bfloat16)
        torch.cuda.synchronize()
        return y, s

    y0, s0 = call()
    for _ in range(4):
        y, s = call()
        assert torch.equal(y, y0) and torch.equal(s, s0)
    for b in range(3):
        y, s = call(slice(b, b + 1))
        assert torch.equal(y, y0[b:b + 1]) and torch.equal(s, s0[b:b + 1])
    assert abi.lib().dc_device_status(1) == 0

"""GPU test of dc_chunk_fwd_noalloc, the entry point that allocates nothing.

Some callers cannot hand this library device scratch: an engine whose device
memory all belongs to its own pool and whose FFI boundary passes only the
inputs and outputs, or a serving loop where cudaMalloc (which can synchronise
the device) must not run.  dc_chunk_fwd_noalloc runs the two-kernel
tensor-core path with its workspace in the library's fixed device array.

Called through the C ABI, each case is compared with dc_chunk_fwd (the same
path over a caller-owned workspace) bit for bit -- the same kernels on the same
inputs must give the same bytes -- and with the float64 oracle on the same
bf16-rounded inputs, within the 2e-2 bf16 bar of the other tensor-core tests,
for two calls in a row with different inputs (the second call reuses the array
the first one left behind).  Cases: per-channel gates (GDN-2) with fp32
output, per-head gates, and bf16 output.  This file is collected last on
purpose, and it runs alone in a fresh process as well as after the others."""
import importlib

import numpy as np
import pytest
import torch

import oracle
from _inputs import config_inputs

pytestmark = pytest.mark.gpu
dn = importlib.import_module("burn-deltanet_b200")
abi = importlib.import_module("burn-deltanet_b200._abi")

TOL = 2e-2  # bf16 q/k/v with fp32 state and accumulation: the north star's bf16 bound


def device_inputs(seed, cfg=5, batch=2, seq=300, heads=4):
    raw = config_inputs(cfg, np.random.default_rng(seed), batch, seq, heads, 128, 128)
    raw["state"] = np.random.default_rng(seed + 1).normal(0, 0.02, raw["state"].shape)
    t = {}
    for name in ("q", "k", "v"):
        t[name] = torch.from_numpy(raw[name]).to("cuda", torch.bfloat16).contiguous()
    for name in ("erase", "write", "g", "state"):
        t[name] = torch.from_numpy(raw[name]).to("cuda", torch.float32).contiguous()
    return t


def chunk_args(t, y, s_out, flags=0):
    a = abi.ChunkArgs()
    b, s, h, dk = t["q"].shape
    a.batch, a.seq, a.heads, a.dk, a.dv = b, s, h, dk, t["v"].shape[3]
    a.n_householder = 1
    a.erase_w, a.write_w, a.g_w = t["erase"].shape[3], t["write"].shape[3], t["g"].shape[3]
    a.chunk_len, a.in_dtype, a.gate_dtype = 64, abi.DC_BF16, abi.DC_F32
    a.out_dtype = abi.DC_BF16 if y.dtype == torch.bfloat16 else abi.DC_F32
    a.flags, a.scale = flags, 1.0 / np.sqrt(dk)
    a.q, a.k, a.v = t["q"].data_ptr(), t["k"].data_ptr(), t["v"].data_ptr()
    a.erase, a.write, a.g = t["erase"].data_ptr(), t["write"].data_ptr(), t["g"].data_ptr()
    a.state_in, a.y, a.state_out = t["state"].data_ptr(), y.data_ptr(), s_out.data_ptr()
    return a


def run(t, noalloc, out_dtype):
    b, s, h, _ = t["q"].shape
    y = torch.full((b, s, h, 128), float("nan"), device="cuda", dtype=out_dtype)
    s_out = torch.full_like(t["state"], float("nan"))
    stream = torch.cuda.current_stream().cuda_stream
    if noalloc:
        st = abi.lib().dc_chunk_fwd_noalloc(chunk_args(t, y, s_out), stream)
    else:
        # per-head gates take the two-kernel path only when asked (they have the fused kernel otherwise)
        a = chunk_args(t, y, s_out, flags=abi.DC_FLAG_FORCE_SPLIT)
        ws = torch.empty(abi.lib().dc_chunk_workspace_size(a), dtype=torch.uint8, device="cuda")
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        assert abi.lib().dc_chunk_kernel_choice(a) == 2
        st = abi.lib().dc_chunk_fwd(a, stream)
    assert st == abi.DC_OK, abi.status_string(st)
    torch.cuda.synchronize()
    return y, s_out


def oracle_ref(t):
    r = {n: t[n].double().cpu().numpy() for n in ("q", "k", "v", "erase", "write", "g", "state")}
    return oracle.householder("recurrent", r["q"], r["k"], r["v"], r["erase"], r["write"], r["g"], r["state"], 1)


@pytest.mark.parametrize("cfg,out_dtype", [
    (5, torch.float32),    # GDN-2: per-channel erase, write and log-decay
    (1, torch.float32),    # per-head beta and log-decay (erase_w = write_w = g_w = 1)
    (5, torch.bfloat16),   # bf16 y leaves through the scan kernel's TMA store
])
def test_noalloc_matches_workspace_entry_point_twice(cfg, out_dtype):
    assert abi.lib().dc_device_status(1) == 0
    for seed in (1, 2):  # two calls in a row share the one scratch array
        t = device_inputs(seed, cfg)
        y_na, s_na = run(t, noalloc=True, out_dtype=out_dtype)
        y_ws, s_ws = run(t, noalloc=False, out_dtype=out_dtype)
        assert torch.isfinite(y_na).all() and torch.isfinite(s_na).all()
        assert torch.equal(y_na, y_ws) and torch.equal(s_na, s_ws), (
            (y_na.float() - y_ws.float()).abs().max().item(), (s_na - s_ws).abs().max().item())
        y_o, s_o = oracle_ref(t)
        ey = np.abs(y_na.double().cpu().numpy() - y_o).max()
        es = np.abs(s_na.double().cpu().numpy() - s_o).max()
        print(f"cfg {cfg} {out_dtype} seed {seed}: max |y - oracle| {ey:.3e}, max |S - oracle| {es:.3e}")
        assert ey < TOL and es < TOL, (ey, es)
    assert abi.lib().dc_device_status(1) == 0


def test_noalloc_rejects_oversized_and_flagged_requests():
    t = device_inputs(3, batch=1, seq=64, heads=1)
    y = torch.empty(1, 64, 1, 128, device="cuda")
    s_out = torch.empty_like(t["state"])
    a = chunk_args(t, y, s_out)
    stream = torch.cuda.current_stream().cuda_stream
    # one chunk past the array: rejected on the host, nothing enqueued
    per_chunk = abi.lib().dc_chunk_workspace_size(a)
    a.heads = abi.DC_NOALLOC_SCRATCH_BYTES // per_chunk + 1
    assert abi.lib().dc_chunk_fwd_noalloc(a, stream) == abi.DC_ESCRATCH
    a.heads = 1
    a.flags = abi.DC_FLAG_RECURRENT
    assert abi.lib().dc_chunk_fwd_noalloc(a, stream) == abi.DC_EINVAL_ARG

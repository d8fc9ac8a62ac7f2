"""GPU test of dc_chunk_fwd_noalloc, the entry point that allocates nothing:
the two-kernel tensor-core path with its workspace in the library's fixed
device array.  Called through the C ABI and compared with dc_chunk_fwd (the
same path over a caller-owned workspace) on the same inputs, for two calls in
a row with different inputs.  This file is collected last on purpose."""
import importlib

import numpy as np
import pytest
import torch

from _inputs import config_inputs

pytestmark = pytest.mark.gpu
dn = importlib.import_module("burn-deltanet_b200")
abi = importlib.import_module("burn-deltanet_b200._abi")

TOL = 2e-2  # the bf16 bar of the other tensor-core tests


def device_inputs(seed, batch=2, seq=300, heads=4):
    raw = config_inputs(5, np.random.default_rng(seed), batch, seq, heads, 128, 128)
    raw["state"] = np.random.default_rng(seed + 1).normal(0, 0.02, raw["state"].shape)
    t = {}
    for name in ("q", "k", "v"):
        t[name] = torch.from_numpy(raw[name]).to("cuda", torch.bfloat16).contiguous()
    for name in ("erase", "write", "g", "state"):
        t[name] = torch.from_numpy(raw[name]).to("cuda", torch.float32).contiguous()
    return t


def chunk_args(t, y, s_out):
    a = abi.ChunkArgs()
    b, s, h, dk = t["q"].shape
    a.batch, a.seq, a.heads, a.dk, a.dv = b, s, h, dk, t["v"].shape[3]
    a.n_householder = 1
    a.erase_w, a.write_w, a.g_w = t["erase"].shape[3], t["write"].shape[3], t["g"].shape[3]
    a.chunk_len, a.in_dtype, a.gate_dtype, a.out_dtype = 64, abi.DC_BF16, abi.DC_F32, abi.DC_F32
    a.flags, a.scale = 0, 1.0 / np.sqrt(dk)
    a.q, a.k, a.v = t["q"].data_ptr(), t["k"].data_ptr(), t["v"].data_ptr()
    a.erase, a.write, a.g = t["erase"].data_ptr(), t["write"].data_ptr(), t["g"].data_ptr()
    a.state_in, a.y, a.state_out = t["state"].data_ptr(), y.data_ptr(), s_out.data_ptr()
    return a


def run(t, noalloc):
    b, s, h, _ = t["q"].shape
    y = torch.full((b, s, h, 128), float("nan"), device="cuda")
    s_out = torch.full_like(t["state"], float("nan"))
    a = chunk_args(t, y, s_out)
    stream = torch.cuda.current_stream().cuda_stream
    if noalloc:
        st = abi.lib().dc_chunk_fwd_noalloc(a, stream)
    else:
        ws = torch.empty(abi.lib().dc_chunk_workspace_size(a), dtype=torch.uint8, device="cuda")
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        assert abi.lib().dc_chunk_kernel_choice(a) == 2
        st = abi.lib().dc_chunk_fwd(a, stream)
    assert st == abi.DC_OK, abi.status_string(st)
    torch.cuda.synchronize()
    return y.double().cpu().numpy(), s_out.double().cpu().numpy()


def test_noalloc_matches_workspace_entry_point_twice():
    assert abi.lib().dc_device_status(1) == 0
    for seed in (1, 2):  # two calls in a row share the one scratch array
        t = device_inputs(seed)
        y_na, s_na = run(t, noalloc=True)
        y_ws, s_ws = run(t, noalloc=False)
        assert np.isfinite(y_na).all() and np.isfinite(s_na).all()
        ey, es = np.abs(y_na - y_ws).max(), np.abs(s_na - s_ws).max()
        print(f"seed {seed}: max |y diff| {ey:.3e}, max |S diff| {es:.3e}")
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

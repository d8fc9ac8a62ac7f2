"""GPU tests of the failure path: a bounded wait that runs out.

Every wait in the kernels is bounded; one that runs out sets the device status
word, lets the CTA's own loads in flight land, frees its tensor memory and
returns.  The DC_FLAG_TEST_STALL hook makes that happen without any fault: the
kernel issues none of its tile loads, so its waits on them run out (about 2 s).
Each test checks that the call reports it through dc_device_status, writes
no output, and leaves the context usable: the same call without the hook,
before and after, gives identical results and a clean status."""
import importlib
import math
import time

import pytest
import torch

pytestmark = pytest.mark.gpu
abi = importlib.import_module("burn-deltanet_b200._abi")

D = 128
WAIT_LIMIT_S = 2.0  # the kernels' bounded-wait limit


def l2n(x):
    return x / torch.sqrt((x * x).sum(-1, keepdim=True) + 1e-6)


def prefill_inputs(batch=1, seq=200, heads=2, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    rn = lambda *s: torch.randn(*s, device="cuda", generator=g)
    beta = torch.sigmoid(rn(batch, seq, heads, 1))
    return dict(q=l2n(rn(batch, seq, heads, D)).bfloat16(), k=l2n(rn(batch, seq, heads, D)).bfloat16(),
                v=rn(batch, seq, heads, D).bfloat16(), erase=beta, write=beta.clone(),
                g=-torch.nn.functional.softplus(rn(batch, seq, heads, 1)),
                state=0.02 * rn(batch, heads, D, D))


def chunk_call(t, flags):
    b, s, h, _ = t["q"].shape
    y = torch.full((b, s, h, D), 7.0, device="cuda")
    s_out = torch.full_like(t["state"], 7.0)
    a = abi.ChunkArgs()
    a.batch, a.seq, a.heads, a.dk, a.dv = b, s, h, D, D
    a.n_householder, a.erase_w, a.write_w, a.g_w, a.chunk_len = 1, 1, 1, 1, 64
    a.in_dtype, a.gate_dtype, a.out_dtype = abi.DC_BF16, abi.DC_F32, abi.DC_F32
    a.flags, a.scale = flags, 1.0 / math.sqrt(D)
    a.q, a.k, a.v = t["q"].data_ptr(), t["k"].data_ptr(), t["v"].data_ptr()
    a.erase, a.write, a.g = t["erase"].data_ptr(), t["write"].data_ptr(), t["g"].data_ptr()
    a.state_in, a.y, a.state_out = t["state"].data_ptr(), y.data_ptr(), s_out.data_ptr()
    assert abi.lib().dc_chunk_kernel_choice(a) == 1  # the tensor-core kernel
    t0 = time.monotonic()
    st = abi.lib().dc_chunk_fwd(a, torch.cuda.current_stream().cuda_stream)
    assert st == abi.DC_OK, abi.status_string(st)
    torch.cuda.synchronize()
    return y, s_out, time.monotonic() - t0


def step_call(t, flags):
    b, h, _ = t["q"].shape
    y = torch.full((b, h, D), 7.0, device="cuda")
    s_out = torch.full_like(t["state"], 7.0)
    a = abi.StepArgs()
    a.batch, a.heads, a.dk, a.dv = b, h, D, D
    a.n_householder, a.erase_w, a.write_w, a.g_w = 1, 1, 1, 1
    a.in_dtype, a.gate_dtype, a.out_dtype = abi.DC_BF16, abi.DC_F32, abi.DC_F32
    a.flags, a.scale = flags, 1.0 / math.sqrt(D)
    a.q, a.k, a.v = t["q"].data_ptr(), t["k"].data_ptr(), t["v"].data_ptr()
    a.erase, a.write, a.g = t["erase"].data_ptr(), t["write"].data_ptr(), t["g"].data_ptr()
    a.state_in, a.y, a.state_out = t["state"].data_ptr(), y.data_ptr(), s_out.data_ptr()
    t0 = time.monotonic()
    st = abi.lib().dc_step(a, torch.cuda.current_stream().cuda_stream)
    assert st == abi.DC_OK, abi.status_string(st)
    torch.cuda.synchronize()
    return y, s_out, time.monotonic() - t0


def check_stall(call, t):
    assert abi.lib().dc_device_status(1) == 0
    y0, s0, _ = call(t, 0)
    assert abi.lib().dc_device_status(0) == 0
    y, s, secs = call(t, abi.DC_FLAG_TEST_STALL)
    assert abi.lib().dc_device_status(1) == 1, "the wait that ran out was not reported"
    assert secs > 0.5 * WAIT_LIMIT_S, f"returned after {secs:.2f} s: the wait did not run to its limit"
    assert bool((y == 7.0).all()) and bool((s == 7.0).all()), "a stalled call wrote output"
    y1, s1, _ = call(t, 0)  # the context is still usable
    assert abi.lib().dc_device_status(1) == 0
    assert torch.equal(y0, y1) and torch.equal(s0, s1)
    assert torch.isfinite(y1).all() and torch.isfinite(s1).all()


def test_prefill_wait_that_runs_out_is_reported_and_the_context_survives():
    check_stall(chunk_call, prefill_inputs())


def test_decode_wait_that_runs_out_is_reported_and_the_context_survives():
    g = torch.Generator(device="cuda").manual_seed(1)
    rn = lambda *s: torch.randn(*s, device="cuda", generator=g)
    b, h = 2, 3
    t = dict(q=l2n(rn(b, h, D)).bfloat16(), k=l2n(rn(b, h, D)).bfloat16(), v=rn(b, h, D).bfloat16(),
             erase=torch.sigmoid(rn(b, h, 1)), write=torch.sigmoid(rn(b, h, 1)),
             g=-torch.nn.functional.softplus(rn(b, h, 1)), state=0.02 * rn(b, h, D, D))
    check_stall(step_call, t)


def test_stall_hook_is_refused_where_it_does_not_apply():
    t = prefill_inputs(seq=64)
    b, s, h, _ = t["q"].shape
    y = torch.empty(b, s, h, D, device="cuda")
    s_out = torch.empty_like(t["state"])
    a = abi.ChunkArgs()
    a.batch, a.seq, a.heads, a.dk, a.dv = b, s, h, D, D
    a.n_householder, a.erase_w, a.write_w, a.g_w, a.chunk_len = 1, 1, 1, 1, 64
    a.in_dtype, a.gate_dtype, a.out_dtype = abi.DC_BF16, abi.DC_F32, abi.DC_F32
    a.flags, a.scale = abi.DC_FLAG_TEST_STALL | abi.DC_FLAG_FORCE_SIMT, 0.1
    a.q, a.k, a.v = t["q"].data_ptr(), t["k"].data_ptr(), t["v"].data_ptr()
    a.erase, a.write, a.g = t["erase"].data_ptr(), t["write"].data_ptr(), t["g"].data_ptr()
    a.state_in, a.y, a.state_out = t["state"].data_ptr(), y.data_ptr(), s_out.data_ptr()
    stream = torch.cuda.current_stream().cuda_stream
    assert abi.lib().dc_chunk_fwd(a, stream) == abi.DC_EINVAL_ARG
    assert abi.lib().dc_chunk_fwd_noalloc(a, stream) == abi.DC_EINVAL_ARG
    assert abi.lib().dc_device_status(0) == 0

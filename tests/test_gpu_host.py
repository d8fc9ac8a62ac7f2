"""GPU tests of dc_chunk_fwd_host, the prefill from host memory.

The entry point streams the batch through the GPU in slices of whole
sequences (copies in, kernels, copies out on three streams, two slices in
flight).  Every kernel path works per (batch, head), so the results must be
bit-identical to dc_chunk_fwd on device copies of the same inputs: the fused
tensor-core kernel, the two-kernel per-channel-gate path (whose workspace the
slices share), the fp32-accurate chunked path and the CUDA-core kernel."""
import importlib
import math

import numpy as np
import pytest
import torch

from _inputs import config_inputs

pytestmark = pytest.mark.gpu
dn = importlib.import_module("burn-deltanet_b200")
abi = importlib.import_module("burn-deltanet_b200._abi")


def host_inputs(cfg, batch, seq, heads, d, u=1, seed=0, in_dtype=torch.bfloat16):
    raw = config_inputs(cfg, np.random.default_rng(seed), batch, seq, heads, d, d, u=u)
    raw["state"] = np.random.default_rng(seed + 1).normal(0, 0.02, raw["state"].shape)
    t = {}
    for name in ("q", "k", "v"):
        t[name] = torch.from_numpy(raw[name]).to(in_dtype).contiguous().pin_memory()
    for name in ("erase", "write", "g", "state"):
        t[name] = None if raw[name] is None else torch.from_numpy(raw[name]).float().contiguous().pin_memory()
    return t


def both(t, u=1, out_dtype=None, **kw):
    d = t["q"].shape[3]
    gated = t["g"] is not None
    dev = {k: (None if v is None else v.cuda()) for k, v in t.items()}
    y_d, s_d = dn.delta_chunk_recalculated(dev["q"], dev["k"], dev["v"], dev["erase"], dev["write"], dev["g"],
                                           dev["state"], gated, 64, 1 / math.sqrt(d), n_householder=u,
                                           out_dtype=out_dtype, **kw)
    torch.cuda.synchronize()
    y_h, s_h = dn.delta_chunk_recalculated_host(t["q"], t["k"], t["v"], t["erase"], t["write"], t["g"],
                                                t["state"], gated, 64, 1 / math.sqrt(d), n_householder=u,
                                                out_dtype=out_dtype, **kw)
    assert y_h.device.type == "cpu" and s_h.device.type == "cpu"
    assert abi.lib().dc_device_status(1) == 0
    return (y_d.cpu(), s_d.cpu()), (y_h, s_h)


@pytest.mark.parametrize("batch", [1, 3, 11])
def test_host_path_equals_device_path_tensor_core(batch):
    t = host_inputs(2, batch, 150, 3, 128)
    (y_d, s_d), (y_h, s_h) = both(t)
    assert torch.equal(y_d, y_h) and torch.equal(s_d, s_h)


def test_host_path_equals_device_path_deltaproduct():
    t = host_inputs(4, 3, 100, 2, 128, u=2)
    (y_d, s_d), (y_h, s_h) = both(t, u=2, out_dtype=torch.float32)
    assert torch.equal(y_d, y_h) and torch.equal(s_d, s_h)


def test_host_path_equals_device_path_per_channel_gates():
    t = host_inputs(5, 10, 130, 2, 128)  # ten sequences: five slices of two share one workspace
    (y_d, s_d), (y_h, s_h) = both(t)
    assert torch.equal(y_d, y_h) and torch.equal(s_d, s_h)


def test_host_path_equals_device_path_cuda_cores():
    t = host_inputs(1, 4, 90, 2, 32, in_dtype=torch.float32)
    (y_d, s_d), (y_h, s_h) = both(t, force_simt=True)
    assert torch.equal(y_d, y_h) and torch.equal(s_d, s_h)


def test_host_path_equals_device_path_fp32_chunked():
    """float32 inputs take the fp32-accurate chunked path on both sides.  The whole batch (160 heads x 4
    value slices) runs its full-width scan on the device, while the host path's slices of three sequences
    (24 heads) run the sliced scan: the two forms give the same bits, so the results still match exactly."""
    t = host_inputs(1, 20, 70, 8, 128, in_dtype=torch.float32)
    (y_d, s_d), (y_h, s_h) = both(t)
    assert torch.equal(y_d, y_h) and torch.equal(s_d, s_h)


def test_host_path_reuses_scratch_and_honours_the_stream():
    t = host_inputs(2, 4, 200, 2, 128, seed=5)
    d = 128
    a_y = torch.empty(4, 200, 2, d, dtype=torch.bfloat16, pin_memory=True)
    a_s = torch.empty(4, 2, d, d, pin_memory=True)
    dev = {k: (None if v is None else v.cuda()) for k, v in t.items()}
    y_d, s_d = dn.delta_chunk_recalculated(dev["q"], dev["k"], dev["v"], dev["erase"], dev["write"], None,
                                           dev["state"], False, 64, 1 / math.sqrt(d))
    scratch = None
    for _ in range(3):  # back to back on one stream, one scratch, outputs rewritten in place
        if scratch is None:
            need = dn.delta_chunk_host_scratch_size(t["q"], t["k"], t["v"], t["erase"], t["write"], None,
                                                    t["state"], False, 64, 1 / math.sqrt(d))
            scratch = torch.empty(need, dtype=torch.uint8, device="cuda")
        a_y.fill_(0)
        dn.delta_chunk_recalculated_host(t["q"], t["k"], t["v"], t["erase"], t["write"], None, t["state"], False,
                                         64, 1 / math.sqrt(d), scratch=scratch, y_out=a_y, state_out=a_s,
                                         synchronize=False)
        torch.cuda.current_stream().synchronize()
        assert torch.equal(a_y, y_d.cpu()) and torch.equal(a_s, s_d.cpu())

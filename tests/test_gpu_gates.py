"""GPU parity of the front-end's gate producers (dc_gates) against the float64 oracle.

The write gates (sigma, 2 sigma; src/common/qkv.rs:333-368), ForgetGate::log_decay (src/common/gate.rs:
51-59, with its clamp) and ChannelForgetGate::log_decay (gate.rs:178-196, after its up projection), on
float32 and bf16 inputs, contiguous and as column slices of a wider projection, with arguments large
enough to reach softplus's linear range and sigma's saturation.  Bar: 1e-5 relative (float32 out)."""
import importlib

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
dn = importlib.import_module("burn-deltanet_b200")


def close(got, ref, tol=1e-5):
    got = got.double().cpu().numpy()
    err = np.abs(got - ref) / np.maximum(1.0, np.abs(ref))
    assert got.shape == ref.shape and err.max() < tol, err.max()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("sliced", [False, True])
def test_write_gates(dtype, sliced):
    g = torch.Generator(device="cuda").manual_seed(1)
    proj = (torch.randn(3, 50, 40, device="cuda", generator=g) * 8).to(dtype)
    raw = proj[:, :, 5:21] if sliced else proj[:, :, :16].contiguous()
    ref_in = raw.double().cpu().numpy()
    close(dn.write_gate(raw, doubled=True), oracle.write_gate(ref_in, True))
    close(dn.write_gate(raw), oracle.write_gate(ref_in, False))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_head_log_decay(dtype):
    g = torch.Generator(device="cuda").manual_seed(2)
    proj = (torch.randn(2, 70, 24, device="cuda", generator=g) * 10).to(dtype)
    dt = proj[:, :, 8:24]
    bias = torch.randn(16, device="cuda", generator=g)
    a = torch.rand(16, device="cuda", generator=g) * np.log(16.0)
    for limit in ((0.0, 6.5504e4), (0.01, 2.0)):
        got = dn.head_log_decay(dt, bias, a, limit)
        close(got, oracle.head_log_decay(dt.double().cpu().numpy(), bias.double().cpu().numpy(),
                                         a.double().cpu().numpy(), limit))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_channel_log_decay(dtype):
    g = torch.Generator(device="cuda").manual_seed(3)
    dt = (torch.randn(2, 33, 4 * 32, device="cuda", generator=g) * 3).to(dtype)
    bias = torch.randn(4 * 32, device="cuda", generator=g)
    a = torch.randn(4, device="cuda", generator=g)
    got = dn.channel_log_decay(dt, bias, a, 32, -5.0)
    close(got, oracle.channel_log_decay(dt.double().cpu().numpy(), bias.double().cpu().numpy(),
                                        a.double().cpu().numpy(), 32, -5.0))

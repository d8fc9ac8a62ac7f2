"""GPU parity of the per-head output normalisation (dc_out_norm) against the float64 oracle.

OutNorm (src/common/norm.rs:106-144) over head_v_dim: gated (y / rms * w * silu(gate)) and plain, bf16 and
float32 in / out, head sizes 128 (the benchmark), 64, and widths that do not fill a warp (7, 40, 200),
zero rows (the epsilon guard) and in place.  Bar: 1e-5 relative for float32 out (fp32 arithmetic),
bf16 rounding (2^-8 of the value) for bf16 out, on the same (rounded) inputs."""
import importlib

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
dn = importlib.import_module("burn-deltanet_b200")
abi = importlib.import_module("burn-deltanet_b200._abi")


def run(shape, gated, in_dtype, out_dtype, eps=1e-5, seed=0, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    y = (torch.randn(*shape, device="cuda", generator=g) * scale).to(in_dtype)
    gate = (torch.randn(*shape, device="cuda", generator=g) * 2).to(in_dtype) if gated else None
    w = torch.rand(shape[-1], device="cuda", generator=g) + 0.5
    out = dn.out_norm(y, gate, w, eps, out_dtype=out_dtype)
    torch.cuda.synchronize()
    ref = oracle.out_norm(y.double().cpu().numpy(), None if gate is None else gate.double().cpu().numpy(),
                          w.double().cpu().numpy(), eps)
    return out.double().cpu().numpy(), ref


@pytest.mark.parametrize("gated", [True, False])
@pytest.mark.parametrize("in_dtype,out_dtype", [(torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32),
                                                (torch.bfloat16, torch.float32), (torch.float32, torch.bfloat16)])
@pytest.mark.parametrize("shape", [(2, 37, 16, 128), (1, 5, 3, 64), (3, 4, 2, 7), (2, 9, 3, 40), (1, 3, 2, 200)])
def test_out_norm_matches_the_oracle(gated, in_dtype, out_dtype, shape):
    got, ref = run(shape, gated, in_dtype, out_dtype, seed=sum(shape))
    tol = 1e-5 if out_dtype == torch.float32 else 2 ** -8
    err = np.abs(got - ref) / np.maximum(1.0, np.abs(ref))
    assert err.max() < tol, err.max()


def test_out_norm_zero_rows_and_large_values():
    got, ref = run((1, 64, 4, 128), True, torch.float32, torch.float32, scale=0.0)
    assert np.array_equal(got, np.zeros_like(got))
    got, ref = run((1, 64, 4, 128), True, torch.float32, torch.float32, scale=1e4, seed=5)
    assert np.abs(got - ref).max() / np.abs(ref).max() < 1e-5


def test_out_norm_in_place_and_many_rows():
    """In place on a config-2-sized output (B=8, T=4096, H=16, dv=128: 524,288 rows, grid-stride loop)."""
    g = torch.Generator(device="cuda").manual_seed(9)
    y = torch.randn(8, 4096, 16, 128, device="cuda", generator=g).to(torch.bfloat16)
    gate = torch.randn(8, 4096, 16, 128, device="cuda", generator=g).to(torch.bfloat16)
    w = torch.rand(128, device="cuda", generator=g) + 0.5
    y0 = y.clone()
    want = dn.out_norm(y, gate, w)
    got = dn.out_norm(y, gate, w, out=y)
    torch.cuda.synchronize()
    assert got.data_ptr() == y.data_ptr() and torch.equal(got, want)
    rows = torch.from_numpy(np.random.default_rng(0).integers(0, 8 * 4096 * 16, 256)).cuda()
    ref = oracle.out_norm(y0.view(-1, 128)[rows].double().cpu().numpy(), gate.view(-1, 128)[rows].double().cpu().numpy(),
                          w.double().cpu().numpy(), 1e-5)
    err = np.abs(got.view(-1, 128)[rows].double().cpu().numpy() - ref) / np.maximum(1.0, np.abs(ref))
    assert err.max() < 2 ** -8
    assert abi.lib().dc_device_status(0) == 0


def test_out_norm_rejects_mismatched_inputs():
    y = torch.zeros(2, 3, 4, 8, device="cuda")
    with pytest.raises(dn.DeltaShapeError):
        dn.out_norm(y, torch.zeros(2, 3, 4, 9, device="cuda"), torch.ones(8, device="cuda"))
    with pytest.raises(dn.DeltaShapeError):
        dn.out_norm(y, None, torch.ones(9, device="cuda"))
    with pytest.raises(dn.DeltaCoreError):
        dn.out_norm(y, torch.zeros(2, 3, 4, 8, device="cuda", dtype=torch.bfloat16), torch.ones(8, device="cuda"))

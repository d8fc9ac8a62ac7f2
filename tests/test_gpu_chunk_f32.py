"""GPU parity of the fp32-accurate chunked prefill (dc_chunk_kernel_choice 3): the reference's own
precision (src/delta/chunk.rs:41-221, chunk_recalculated/forward.rs:154-439 in f32) on the tensor cores.

Held to the north star's 1e-4 relative for the fp32 path against the float64 oracle, on the shapes this
path takes (any dk, dv <= 128, a log-decay per head or none, any erase / write width, u >= 1), with
ragged chunk tails, widths that are not multiples of 8, several value slices, long sequences (128
chunks), bf16 inputs (checked on the same rounded inputs) and outputs, in-place state updates, repeat
calls bit for bit, and agreement with the CUDA-core kernel (DC_FLAG_FORCE_SIMT)."""
import importlib
import math

import numpy as np
import pytest
import torch

import oracle
from _inputs import config_inputs, random_raw

pytestmark = pytest.mark.gpu
dn = importlib.import_module("burn-deltanet_b200")
core = importlib.import_module("burn-deltanet_b200.core")
abi = importlib.import_module("burn-deltanet_b200._abi")

F32_TOL = 1e-4


def to_dev(x, dtype=torch.float32):
    return None if x is None else torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


def rel_err(got, want):
    return np.abs(got.double().cpu().numpy() - want).max() / max(1.0, np.abs(want).max())


def dev_inputs(raw, in_dtype=torch.float32):
    d = {n: to_dev(raw[n], in_dtype if n in ("q", "k", "v") else torch.float32)
         for n in ("q", "k", "v", "erase", "write", "g")}
    d["state"] = to_dev(raw["state"])
    return d


def choice(d, u, out_dtype=torch.float32, force_simt=False):
    """The kernel dc_chunk_fwd takes for these tensors, with the workspace the Python layer passes."""
    gated = d["g"] is not None
    a, _, _ = core._chunk_args(d["q"], d["k"], d["v"], d["erase"], d["write"], d["g"], d["state"], gated, 64, 0.5, u,
                               out_dtype, force_simt, False, False, None, None, core._check_tensor,
                               lambda shape, dt: torch.empty(shape, device="cuda", dtype=dt))
    need = abi.lib().dc_chunk_workspace_size(a)
    a.workspace, a.workspace_bytes = (0x100000 if need else None), need
    return abi.lib().dc_chunk_kernel_choice(a)


def run(d, u, out_dtype=torch.float32, force_simt=False, state_out=None):
    scale = 1.0 / math.sqrt(d["q"].shape[3])
    return dn.delta_chunk_recalculated(d["q"], d["k"], d["v"], d["erase"], d["write"], d["g"], d["state"],
                                       d["g"] is not None, 64, scale, n_householder=u, out_dtype=out_dtype,
                                       force_simt=force_simt, state_out=state_out)


def oracle_of(d, u):
    n = {k: None if t is None else t.double().cpu().numpy() for k, t in d.items()}
    return oracle.householder("recurrent", n["q"], n["k"], n["v"], n["erase"], n["write"], n["g"], n["state"], u)


CASES = [
    # b, s, h, dk, dv, u, gated, full-width erase / write, random S0
    (2, 200, 3, 128, 128, 1, True, False, True),     # 7 chunks, the last partial
    (1, 500, 2, 64, 64, 1, True, False, True),       # config 1's head size
    (2, 97, 2, 5, 7, 1, False, False, False),        # widths that are not multiples of 8
    (1, 150, 2, 40, 100, 2, True, True, True),       # u = 2, full-width gates, four value slices
    (1, 45, 2, 32, 32, 3, True, False, True),        # u = 3
    (1, 1, 1, 16, 16, 1, True, False, True),         # one token
    (1, 33, 2, 128, 40, 1, False, True, True),       # ungated, a 40-column slice tail
    (1, 4096, 1, 128, 128, 1, True, False, True),    # 128 chunks of state carried
    # more (head, 32-column slice) pairs than two per SM: the full-width scan (one CTA per head)
    (8, 150, 10, 128, 128, 1, True, False, True),
    (10, 70, 10, 40, 72, 2, True, True, True),       # partial warp tiles in both of its products
    (16, 64, 6, 128, 128, 1, False, False, False),
]


@pytest.mark.parametrize("b,s,h,dk,dv,u,gated,full,rs", CASES)
def test_chunked_fp32_matches_the_oracle(b, s, h, dk, dv, u, gated, full, rs):
    rng = np.random.default_rng(300 + s + dk + u)
    raw = random_raw(rng, b, s * u, h, dk, dv, 1.5 if u > 1 else 0.95, gated, rs, full)
    # fold: q and g once per token
    raw["q"], raw["g"] = raw["q"][:, :s], None if raw["g"] is None else raw["g"][:, :s, :, :1]
    d = dev_inputs(raw)
    assert choice(d, u) == 3
    pairs = b * h * (((dv + 7) // 8 * 8 + 31) // 32)
    wide = pairs > 2 * torch.cuda.get_device_properties(0).multi_processor_count
    assert abi.lib().dc_device_status(1) == 0
    y, st = run(d, u)
    torch.cuda.synchronize()
    y0, s0 = oracle_of(d, u)
    ey, es = rel_err(y, y0), rel_err(st, s0)
    print(f"b={b} s={s} h={h} dk={dk} dv={dv} u={u} ({'full-width' if wide else 'sliced'} scan): y {ey:.2e} S {es:.2e}")
    assert ey < F32_TOL and es < F32_TOL
    assert abi.lib().dc_device_status(1) == 0


def test_config1_recipe_takes_the_chunked_path():
    """Config 1 (GDN core, fp32, B=2 T=512 H=4 d=64, per-head gate) now runs on the tensor cores."""
    raw = config_inputs(1, np.random.default_rng(0), 2, 512, 4, 64, 64)
    d = dev_inputs(raw)
    assert choice(d, 1) == 3
    y, st = run(d, 1)
    y0, s0 = oracle_of(d, 1)
    assert rel_err(y, y0) < F32_TOL and rel_err(st, s0) < F32_TOL


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_bf16_inputs_on_the_chunked_path(out_dtype):
    """bf16 q/k/v at d = 64 (not the fused kernel's shape): fp32-accurate on the rounded inputs."""
    raw = config_inputs(4, np.random.default_rng(8), 2, 150, 3, 64, 64, u=2)
    raw["state"] = np.random.default_rng(9).normal(0, 0.05, (2, 3, 64, 64))
    d = dev_inputs(raw, torch.bfloat16)
    assert choice(d, 2, out_dtype) == 3
    y, st = run(d, 2, out_dtype)
    y0, s0 = oracle_of(d, 2)
    assert y.dtype == out_dtype
    assert rel_err(st, s0) < F32_TOL
    assert rel_err(y, y0) < (F32_TOL if out_dtype == torch.float32 else 2 ** -8)


@pytest.mark.parametrize("b,h", [(2, 2), (20, 4)])  # the sliced and the full-width scan
def test_chunked_agrees_with_the_cuda_core_kernel_and_repeats_bit_for_bit(b, h):
    raw = config_inputs(1, np.random.default_rng(4), b, 300, h, 128, 128)
    raw["state"] = np.random.default_rng(5).normal(0, 0.05, (b, h, 128, 128))
    d = dev_inputs(raw)
    assert choice(d, 1, force_simt=True) == 0
    y1, s1 = run(d, 1)
    y2, s2 = run(d, 1)
    ys, ss = run(d, 1, force_simt=True)
    st = d["state"].clone()
    d_in = dict(d, state=st)
    y3, s3 = run(d_in, 1, state_out=st)  # in place: the state buffer is read and then overwritten
    torch.cuda.synchronize()
    assert torch.equal(y1, y2) and torch.equal(s1, s2)
    assert torch.equal(y1, y3) and torch.equal(s1, st)
    e = max((y1 - ys).abs().max().item() / max(1.0, ys.abs().max().item()),
            (s1 - ss).abs().max().item() / max(1.0, ss.abs().max().item()))
    assert e < F32_TOL, e
    assert abi.lib().dc_device_status(1) == 0


def test_full_width_and_sliced_scans_give_the_same_bits():
    """The batch runs the full-width scan (80 heads x 4 slices > two per SM), its first two sequences alone
    the sliced one: the same arithmetic in the same order, so y and the state agree bit for bit (the
    batch x head sharding relies on a batch subset matching its rows of the whole batch)."""
    raw = config_inputs(1, np.random.default_rng(12), 10, 150, 8, 128, 128)
    raw["state"] = np.random.default_rng(13).normal(0, 0.05, (10, 8, 128, 128))
    d = dev_inputs(raw)
    sub = {k: None if v is None else v[:2].contiguous() for k, v in d.items()}
    y, st = run(d, 1)
    y2, st2 = run(sub, 1)
    torch.cuda.synchronize()
    assert torch.equal(y[:2], y2) and torch.equal(st[:2], st2)

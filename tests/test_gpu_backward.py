"""GPU parity of the backward (dc_chunk_bwd) against the float64 oracle.

The oracle (oracle/backward.py) is pinned to torch autograd of the recurrence
(tests/test_oracle_backward.py).  Shapes and gate widths are the reference's
own backward tests (src/delta/chunk_recalculated/tests.rs:203-313: ungated,
per head, per channel, beta up to 1.95, partial chunks, dk != dv, a non-zero
incoming state), plus d = 128 and micro-steps.  Bar: the reference's 1e-4 on
every gradient for float32 inputs (relative to the gradient's scale above 1);
bf16 q/k/v are compared on the same rounded inputs."""
import importlib
import zlib

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
dn = importlib.import_module("burn-deltanet_b200")
abi = importlib.import_module("burn-deltanet_b200._abi")

NAMES = ("d_q", "d_k", "d_v", "d_erase", "d_write", "d_g", "d_state")


def make(seed, b, t, h, dk, dv, u, gates, beta_max):
    rng = np.random.default_rng(seed)
    chan = gates == "channel"
    kw, vw = (dk, dv) if chan else (1, 1)
    l2 = lambda x: x / np.sqrt((x * x).sum(-1, keepdims=True) + 1e-6)
    return dict(q=l2(rng.standard_normal((b, t, h, dk))), k=l2(rng.standard_normal((b, t * u, h, dk))),
                v=rng.standard_normal((b, t * u, h, dv)),
                e=rng.uniform(0.05, beta_max, (b, t * u, h, kw)), w=rng.uniform(0.05, 1.0, (b, t * u, h, vw)),
                g=None if gates == "none" else rng.uniform(-0.5, -0.01, (b, t, h, kw)),
                s0=rng.normal(0, 0.2, (b, h, dk, dv)), dy=rng.standard_normal((b, t, h, dv)),
                dsf=rng.standard_normal((b, h, dk, dv)))


def gpu_grads(x, u, in_dtype=torch.float32, with_dsf=True, recurrent=False):
    dev = lambda a, dt=torch.float32: None if a is None else torch.tensor(a, dtype=dt, device="cuda")
    q, k, v = (dev(x[n], in_dtype) for n in ("q", "k", "v"))
    dk = q.shape[3]
    out = dn.delta_chunk_recalculated_backward(dev(x["dy"]), dev(x["dsf"]) if with_dsf else None, q, k, v,
                                               dev(x["e"]), dev(x["w"]), dev(x["g"]), dev(x["s0"]),
                                               x["g"] is not None, 64, 1 / np.sqrt(dk), n_householder=u,
                                               recurrent=recurrent)
    torch.cuda.synchronize()
    assert abi.lib().dc_device_status(1) == 0
    rounded = {n: (t.double().cpu().numpy() if t is not None else None) for n, t in zip(("q", "k", "v"), (q, k, v))}
    return dict(zip(NAMES, (None if t is None else t.double().cpu().numpy() for t in out))), rounded


def check(x, u, in_dtype=torch.float32, tol=1e-4, with_dsf=True, recurrent=False):
    got, r = gpu_grads(x, u, in_dtype, with_dsf, recurrent)
    dk = x["q"].shape[3]
    ref = oracle.recurrent_backward(r["q"], r["k"], r["v"], x["e"], x["w"], x["g"], x["s0"], x["dy"],
                                    x["dsf"] if with_dsf else None, 1 / np.sqrt(dk), u)
    worst = 0.0
    for n in NAMES:
        if ref[n] is None:
            assert got[n] is None
            continue
        assert got[n].shape == ref[n].shape, (n, got[n].shape, ref[n].shape)
        err = np.abs(got[n] - ref[n]).max() / max(1.0, np.abs(ref[n]).max())
        worst = max(worst, err)
        assert err < tol, (n, err)
    return worst


@pytest.mark.parametrize("gates,u,beta_max,dims", [
    ("none", 1, 0.95, (2, 16, 3, 8, 8)),         # tests.rs: matches_the_taped_path_ungated
    ("head", 1, 0.95, (2, 16, 3, 8, 8)),         # ..._per_head_gate
    ("channel", 1, 0.95, (2, 16, 3, 8, 8)),      # ..._per_channel_gates
    ("channel", 1, 0.95, (2, 40, 2, 8, 8)),
    ("head", 1, 1.95, (2, 12, 2, 8, 8)),         # ..._with_negative_eigenvalues
    ("channel", 1, 1.95, (2, 12, 2, 8, 8)),
    ("head", 1, 0.95, (2, 13, 2, 8, 8)),         # ..._with_a_partial_last_chunk
    ("none", 1, 0.95, (1, 5, 1, 4, 4)),
    ("channel", 1, 0.95, (2, 37, 2, 4, 6)),
    ("head", 1, 0.95, (2, 16, 2, 8, 16)),        # ..._with_expanded_values
    ("channel", 1, 0.95, (2, 16, 2, 16, 8)),
    ("head", 2, 1.95, (2, 9, 2, 8, 8)),          # micro-steps (DeltaProduct)
    ("channel", 3, 0.95, (1, 7, 2, 8, 8)),
])
def test_backward_matches_the_oracle(gates, u, beta_max, dims):
    x = make(zlib.crc32(repr((gates, u, beta_max, dims)).encode()), *dims, u, gates, beta_max)
    check(x, u)


def test_backward_without_a_final_state_gradient():
    x = make(5, 2, 20, 2, 8, 8, 1, "head", 0.95)
    check(x, 1, with_dsf=False)


@pytest.mark.parametrize("gates", ["head", "channel"])
def test_backward_d128_bf16_inputs(gates):
    """dk = dv = 128 (the benchmark head size), bf16 q/k/v, 150 tokens (ten checkpoint blocks)."""
    x = make(7, 2, 150, 2, 128, 128, 1, gates, 0.95)
    x["s0"] *= 0.1
    print(f"worst relative error {check(x, 1, torch.bfloat16):.2e}")


def test_autograd_function_trains_through_the_op():
    """DeltaChunkFunction: the forward through dc_chunk_fwd, the gradients through dc_chunk_bwd."""
    x = make(9, 2, 30, 2, 16, 16, 1, "channel", 0.95)
    tt = {n: torch.tensor(x[n], dtype=torch.float32, device="cuda", requires_grad=True)
          for n in ("q", "k", "v", "e", "w", "g", "s0")}
    y, s = dn.DeltaChunkFunction.apply(tt["q"], tt["k"], tt["v"], tt["e"], tt["w"], tt["g"], tt["s0"], True, 64,
                                       0.25, 1)
    loss = (y * torch.tensor(x["dy"], dtype=torch.float32, device="cuda")).sum() + \
        (s * torch.tensor(x["dsf"], dtype=torch.float32, device="cuda")).sum()
    loss.backward()
    ref = oracle.recurrent_backward(x["q"], x["k"], x["v"], x["e"], x["w"], x["g"], x["s0"], x["dy"], x["dsf"],
                                    0.25, 1)
    for n, key in zip(NAMES, ("q", "k", "v", "e", "w", "g", "s0")):
        g = tt[key].grad.double().cpu().numpy()
        assert np.abs(g - ref[n]).max() / max(1.0, np.abs(ref[n]).max()) < 1e-4, n


def test_backward_is_deterministic():
    x = make(11, 3, 40, 2, 32, 32, 1, "channel", 0.95)
    a, _ = gpu_grads(x, 1)
    for _ in range(2):
        b, _ = gpu_grads(x, 1)
        for n in NAMES:
            assert np.array_equal(a[n], b[n]), n


def make_widths(seed, b, t, h, dk, dv, u, gates, beta_max, ew, ww):
    """`make` with the erase / write gates at the given widths (1 or full) and g per head or none."""
    x = make(seed, b, t, h, dk, dv, u, gates, beta_max)
    rng = np.random.default_rng(seed + 1)
    x["e"] = rng.uniform(0.05, beta_max, (b, t * u, h, ew))
    x["w"] = rng.uniform(0.05, 1.0, (b, t * u, h, ww))
    return x


@pytest.mark.parametrize("gates,u,beta_max,dims", [
    ("none", 1, 0.95, (2, 16, 3, 8, 8)),
    ("head", 1, 1.95, (2, 12, 2, 8, 8)),
    ("head", 2, 1.95, (2, 9, 2, 8, 8)),
    ("head", 1, 0.95, (2, 16, 2, 8, 16)),
])
def test_recurrent_backward_still_serves_per_head_gates(gates, u, beta_max, dims):
    """DC_FLAG_RECURRENT sends a per-head (or no) log-decay down the token-by-token backward too."""
    x = make(zlib.crc32(repr(("rec", gates, u, dims)).encode()), *dims, u, gates, beta_max)
    check(x, u, recurrent=True)


@pytest.mark.parametrize("t,u", [(31, 1), (32, 1), (33, 1), (64, 1), (65, 1), (16, 2), (17, 2), (11, 3)])
def test_chunked_backward_at_chunk_boundaries(t, u):
    """Sequences ending just before, on and after a 32-micro-step chunk boundary."""
    x = make(zlib.crc32(repr(("edge", t, u)).encode()), 2, t, 2, 16, 16, u, "head", 1.95)
    check(x, u)


@pytest.mark.parametrize("dk,dv,ew,ww", [
    (8, 40, 1, 1),      # two value slices, the second one partial
    (12, 100, 12, 100),  # full-width erase and write, dk and dv not powers of two
    (128, 64, 1, 64),
    (64, 128, 64, 1),   # four value slices
    (5, 7, 5, 7),       # widths that are not multiples of 4 (zero-padded columns)
])
def test_chunked_backward_head_sizes_and_gate_widths(dk, dv, ew, ww):
    x = make_widths(zlib.crc32(repr(("dims", dk, dv, ew, ww)).encode()), 2, 45, 2, dk, dv, 1, "head", 0.95, ew, ww)
    x["s0"] *= 0.3
    check(x, 1)


@pytest.mark.parametrize("u", [1, 2])
def test_chunked_backward_d128_long(u):
    """dk = dv = 128, 300 tokens (ten chunks at u = 1), per-head gates, bf16 q/k/v."""
    x = make(21 + u, 2, 300, 2, 128, 128, u, "head", 0.95)
    x["s0"] *= 0.1
    print(f"worst relative error {check(x, u, torch.bfloat16):.2e}")


def test_chunked_backward_is_deterministic():
    x = make(12, 3, 70, 2, 32, 48, 1, "head", 0.95)
    a, _ = gpu_grads(x, 1)
    for _ in range(2):
        b, _ = gpu_grads(x, 1)
        for n in NAMES:
            if a[n] is not None:
                assert np.array_equal(a[n], b[n]), n


def test_chunked_and_recurrent_backward_agree():
    """The two CUDA backwards on the same inputs (ungated DeltaNet at d = 128, the benchmark's head size)."""
    x = make(13, 1, 200, 2, 128, 128, 1, "none", 0.95)
    a, _ = gpu_grads(x, 1)
    b, _ = gpu_grads(x, 1, recurrent=True)
    for n in NAMES:
        if a[n] is not None:
            err = np.abs(a[n] - b[n]).max() / max(1.0, np.abs(b[n]).max())
            assert err < 1e-4, (n, err)


def _slice(x, n):
    """The first n sequences of a `make` case."""
    return {k: (None if v is None else v[:n]) for k, v in x.items()}


def test_full_width_scan_matches_the_oracle_and_the_sliced_scan_bit_for_bit():
    """80 heads x 4 value slices exceed two CTAs per SM, so the scan takes its full-width form (one 16-warp
    CTA per head); the first two sequences alone (16 heads) take the sliced form.  Every gradient of those
    sequences must agree bit for bit, and the full batch must meet the oracle."""
    x = make(31, 10, 70, 8, 128, 128, 1, "head", 0.95)
    x["s0"] *= 0.1
    assert 10 * 8 * 4 > 2 * torch.cuda.get_device_properties(0).multi_processor_count
    full, _ = gpu_grads(x, 1)
    part, _ = gpu_grads(_slice(x, 2), 1)
    for n in NAMES:
        if full[n] is not None:
            assert np.array_equal(full[n][:2], part[n]), n
    print(f"worst relative error {check(x, 1):.2e}")

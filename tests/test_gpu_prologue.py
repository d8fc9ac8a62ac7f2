"""GPU parity of the front-end prologue (dc_qkv_prologue) against the float64 oracle (oracle/prologue.py).

The short convolution with its window, the activations, the q / k L2 norm and the micro-step reshape
(src/common/conv.rs, src/common/qkv.rs:373-500), over both kernels (two channels per thread for even head
widths, one for odd widths or outputs that are not 16-byte aligned), the benchmark head size
(dk = dv = 128), sequences
that end inside and on a 32-token tile, a single-token step from a window, DeltaProduct micro-steps
(u = 2, 3), K = 1 (no window), SiLU not fused into the convolution, no norm, x as a column slice of a wider
projection, bf16 and float32.  Split calls carrying the window equal one call, and token-by-token steps
equal the forward (the reference's own split-call property).  Bar: 1e-5 relative for float32 out, bf16
rounding for bf16 out, on the same (rounded) inputs."""
import importlib

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
dn = importlib.import_module("burn-deltanet_b200")
abi = importlib.import_module("burn-deltanet_b200._abi")


def make(seed, b, s, h, dk, dv, u, k, dtype, extra=0, window=True, bias=True):
    g = torch.Generator(device="cuda").manual_seed(seed)
    c = h * dk * (1 + u) + u * h * dv
    proj = torch.randn(b, s, c + extra, device="cuda", generator=g).to(dtype)
    x = proj[:, :, :c] if extra else proj
    w = (torch.randn(c, k, device="cuda", generator=g) * 0.5)
    bias_t = torch.randn(c, device="cuda", generator=g) * 0.1 if bias else None
    win = torch.randn(b, c, k, device="cuda", generator=g) if window else None
    return x, w, bias_t, win


def check(x, h, dk, dv, u, w, bias, win, out_dtype=None, **flags):
    got = dn.qkv_prologue(x, h, dk, dv, w, bias, win, n_householder=u, out_dtype=out_dtype, **flags)
    torch.cuda.synchronize()
    cpu = lambda t: None if t is None else t.double().cpu().numpy()
    ref = oracle.qkv_prologue(cpu(x), h, dk, dv, u, cpu(w), cpu(bias), cpu(win),
                              conv_silu=flags.get("conv_silu", True), qk_silu=flags.get("qk_silu", False),
                              l2=flags.get("l2", True))
    tol = 1e-5 if (out_dtype or x.dtype) == torch.float32 else 2 ** -8
    for name, a, r in zip(("q", "k", "v"), got[:3], ref[:3]):
        assert a.shape == r.shape, name
        err = np.abs(cpu(a) - r) / np.maximum(1.0, np.abs(r))
        assert err.max() < tol, (name, err.max())
    assert np.abs(cpu(got[3]) - ref[3]).max() < 1e-6  # the window carries the inputs exactly
    return got


@pytest.mark.parametrize("s", [1, 31, 32, 33, 70])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_prologue_benchmark_heads(s, dtype):
    x, w, bias, win = make(s, 2, s, 2, 128, 128, 1, 4, dtype)
    check(x, 2, 128, 128, 1, w, bias, win)


@pytest.mark.parametrize("u,dk,dv,k", [(2, 64, 32, 3), (3, 16, 24, 4), (1, 40, 8, 1), (2, 8, 8, 8),
                                      (1, 9, 7, 4), (2, 5, 6, 3)])  # odd widths: one channel per thread
def test_prologue_micro_steps_and_widths(u, dk, dv, k):
    x, w, bias, win = make(u * 100 + dk, 2, 37, 3, dk, dv, u, k, torch.float32, window=k > 1)
    check(x, 3, dk, dv, u, w, bias, win)


def test_prologue_activation_outside_the_convolution_and_no_norm():
    x, w, bias, win = make(5, 1, 40, 2, 32, 32, 2, 4, torch.float32)
    check(x, 2, 32, 32, 2, w, bias, win, conv_silu=False, qk_silu=True)
    check(x, 2, 32, 32, 2, w, bias, win, conv_silu=False, qk_silu=False, l2=False)


def test_prologue_on_a_slice_of_the_whole_projection():
    """x is the first C channels of a wider [B, S, C + gates] projection (token stride > C)."""
    x, w, bias, win = make(6, 2, 45, 2, 64, 64, 1, 4, torch.bfloat16, extra=37)
    assert x.stride(1) > x.shape[2]
    check(x, 2, 64, 64, 1, w, None, win, out_dtype=torch.float32)


def test_split_calls_and_steps_equal_one_call():
    x, w, bias, win = make(7, 2, 50, 2, 32, 32, 1, 4, torch.float32)
    full = dn.qkv_prologue(x, 2, 32, 32, w, bias, win)
    a = dn.qkv_prologue(x[:, :19].contiguous(), 2, 32, 32, w, bias, win)
    b = dn.qkv_prologue(x[:, 19:].contiguous(), 2, 32, 32, w, bias, a[3])
    for i in range(3):
        assert torch.allclose(torch.cat([a[i], b[i]], 1), full[i], rtol=1e-6, atol=1e-6)
    assert torch.equal(b[3], full[3])
    window, outs = win, []
    for t in range(6):
        o = dn.qkv_prologue(x[:, t:t + 1].contiguous(), 2, 32, 32, w, bias, window)
        outs.append(o)
        window = o[3]
    for i in range(3):
        assert torch.allclose(torch.cat([o[i] for o in outs], 1), full[i][:, :6], rtol=1e-6, atol=1e-6)
    assert abi.lib().dc_device_status(0) == 0


def test_prologue_outputs_not_16_byte_aligned():
    """Outputs at an odd element offset take the one-channel kernel (the paired one stores channel pairs)."""
    x, w, bias, win = make(8, 1, 40, 2, 32, 32, 1, 4, torch.float32)
    want = dn.qkv_prologue(x, 2, 32, 32, w, bias, win)
    a = abi.PrologueArgs()
    b_, s_ = x.shape[0], x.shape[1]
    c = 2 * 32 * 2 + 2 * 32
    store = torch.empty(3 * b_ * s_ * 2 * 32 + 3, device="cuda")
    q, k, v = (store[1 + i * b_ * s_ * 64:1 + (i + 1) * b_ * s_ * 64].view(b_, s_, 2, 32) for i in range(3))
    nxt = torch.empty(b_, c, 4, device="cuda")
    a.batch, a.seq, a.heads, a.dk, a.dv, a.n_householder, a.conv_kernel = b_, s_, 2, 32, 32, 1, 4
    a.in_dtype = a.out_dtype = abi.DC_F32
    a.flags = abi.DC_PROLOGUE_CONV_SILU | abi.DC_PROLOGUE_L2
    a.x_stride = x.stride(1)
    a.x, a.conv_weight, a.conv_bias, a.window_in, a.window_out = x.data_ptr(), w.data_ptr(), bias.data_ptr(), win.data_ptr(), nxt.data_ptr()
    a.q, a.k, a.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    assert q.data_ptr() % 16 != 0
    assert abi.lib().dc_qkv_prologue(a, torch.cuda.current_stream().cuda_stream) == abi.DC_OK
    torch.cuda.synchronize()
    for got, ref in zip((q, k, v, nxt), want):
        assert torch.allclose(got, ref, rtol=1e-6, atol=1e-6)

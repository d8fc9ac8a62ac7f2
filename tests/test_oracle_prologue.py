"""The front-end oracle (oracle/prologue.py) against independent implementations and its own invariants.

* the convolution against torch's depthwise conv1d on the window-padded input (conv.rs: Valid padding over
  [window tail | x]), the L2 norm against torch.nn.functional.normalize's definition with the additive eps;
* split calls carrying the window == one call (the reference's split-call property, conv.rs:81-118);
* token-by-token step() == forward (conv.rs:124-160 is the forward at S = 1)."""
import numpy as np
import torch

import oracle


def inputs(seed, b, s, h, dk, dv, u, k):
    rng = np.random.default_rng(seed)
    c = h * dk * (1 + u) + u * h * dv
    return (rng.standard_normal((b, s, c)), rng.standard_normal((c, k)) * 0.5, rng.standard_normal(c) * 0.1,
            rng.standard_normal((b, c, k)))


def test_convolution_and_norm_match_torch():
    x, w, bias, win = inputs(0, 2, 11, 2, 8, 6, 2, 4)
    q, k, v, nxt = oracle.qkv_prologue(x, 2, 8, 6, 2, w, bias, win, conv_silu=True, l2=True)
    pad = torch.cat([torch.from_numpy(win[:, :, 1:]), torch.from_numpy(x).transpose(1, 2)], 2)
    y = torch.nn.functional.conv1d(pad, torch.from_numpy(w)[:, None, :], torch.from_numpy(bias), groups=w.shape[0])
    y = torch.nn.functional.silu(y).transpose(1, 2)
    qt = y[:, :, :16].reshape(2, 11, 2, 8)
    qt = qt / torch.sqrt((qt * qt).sum(-1, keepdim=True) + 1e-6)
    vt = y[:, :, 16 + 32:].reshape(2, 22, 2, 6)
    assert np.abs(q - qt.numpy()).max() < 1e-12 and np.abs(v - vt.numpy()).max() < 1e-12
    assert np.array_equal(nxt, pad[:, :, -4:].numpy())


def test_split_calls_equal_one_call():
    x, w, bias, win = inputs(1, 2, 13, 2, 8, 8, 1, 4)
    full = oracle.qkv_prologue(x, 2, 8, 8, 1, w, bias, win)
    a = oracle.qkv_prologue(x[:, :5], 2, 8, 8, 1, w, bias, win)
    b = oracle.qkv_prologue(x[:, 5:], 2, 8, 8, 1, w, bias, a[3])
    for i in range(3):
        assert np.abs(np.concatenate([a[i], b[i]], 1) - full[i]).max() < 1e-12
    assert np.array_equal(b[3], full[3])


def test_steps_equal_the_forward():
    x, w, bias, win = inputs(2, 1, 6, 1, 4, 4, 3, 3)
    full = oracle.qkv_prologue(x, 1, 4, 4, 3, w, None, win, conv_silu=False, qk_silu=True)
    window, outs = win, []
    for t in range(6):
        o = oracle.qkv_prologue(x[:, t:t + 1], 1, 4, 4, 3, w, None, window, conv_silu=False, qk_silu=True)
        outs.append(o)
        window = o[3]
    for i in range(3):
        assert np.abs(np.concatenate([o[i] for o in outs], 1) - full[i]).max() < 1e-12
    assert np.array_equal(window, full[3])


def test_gate_producers_match_torch():
    """softplus, the sigma / 2 sigma write gates and both log-decays against torch's own functions."""
    rng = np.random.default_rng(9)
    x = rng.standard_normal((5, 12)) * 30  # large arguments: the overflow-free softplus
    assert np.abs(oracle.softplus(x) - torch.nn.functional.softplus(torch.from_numpy(x), threshold=1e9).numpy()).max() < 1e-12
    assert np.abs(oracle.write_gate(x, True) - 2 * torch.sigmoid(torch.from_numpy(x)).numpy()).max() < 1e-15
    dt, bias, a = rng.standard_normal((3, 7, 4)), rng.standard_normal(4), rng.uniform(0, 2.7, 4)
    ref = torch.clamp(torch.nn.functional.softplus(torch.from_numpy(dt + bias)), 0.0, 1.5) * -torch.exp(torch.from_numpy(a))
    assert np.abs(oracle.head_log_decay(dt, bias, a, (0.0, 1.5)) - ref.numpy()).max() < 1e-12
    dt = rng.standard_normal((3, 7, 4 * 5))
    bias = rng.standard_normal(20)
    ref = torch.sigmoid(torch.from_numpy(dt + bias).reshape(3, 7, 4, 5) * torch.exp(torch.from_numpy(a))[:, None]) * -5.0
    assert np.abs(oracle.channel_log_decay(dt, bias, a, 5, -5.0) - ref.numpy()).max() < 1e-12

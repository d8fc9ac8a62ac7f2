"""The backward oracle against torch autograd of the recurrence (CPU, float64).

The reference pins its hand-written backward to autodiff of its own forward
(src/delta/chunk_recalculated/tests.rs:203-313, tolerance 1e-4): this pins the
oracle the GPU backward is checked against the same way, at the reference's
test shapes and gate widths (ungated, per head, per channel, beta up to 1.95,
dk != dv, non-zero incoming state, micro-steps)."""
import zlib

import numpy as np
import pytest
import torch

import oracle


def forward_torch(q, k, v, e, w, g, s0, scale, u):
    b, t, h, dk = q.shape
    dv = v.shape[3]
    S = s0
    ys = []
    for n in range(t * u):
        tok, m = divmod(n, u)
        if g is not None and m == 0:
            S = torch.exp(g[:, tok]).expand(b, h, dk)[..., None] * S
        bk = e[:, n].expand(b, h, dk) * k[:, n]
        un = w[:, n].expand(b, h, dv) * v[:, n] - torch.einsum("bhij,bhi->bhj", S, bk)
        S = S + k[:, n][..., None] * un[:, :, None, :]
        if m == u - 1:
            ys.append(torch.einsum("bhij,bhi->bhj", S, scale * q[:, tok]))
    return torch.stack(ys, dim=1), S


def make(rng, b, t, h, dk, dv, u, gates, beta_max):
    chan = gates == "channel"
    kw, vw = (dk, dv) if chan else (1, 1)
    l2 = lambda x: x / np.sqrt((x * x).sum(-1, keepdims=True) + 1e-6)
    x = dict(q=l2(rng.standard_normal((b, t, h, dk))), k=l2(rng.standard_normal((b, t * u, h, dk))),
             v=rng.standard_normal((b, t * u, h, dv)),
             e=rng.uniform(0.05, beta_max, (b, t * u, h, kw)), w=rng.uniform(0.05, 1.0, (b, t * u, h, vw)),
             g=None if gates == "none" else rng.uniform(-0.5, -0.01, (b, t, h, kw)),
             s0=rng.normal(0, 0.2, (b, h, dk, dv)))
    return x


@pytest.mark.parametrize("gates,u,beta_max,dims", [
    ("none", 1, 0.95, (2, 16, 3, 8, 8)),
    ("head", 1, 0.95, (2, 16, 3, 8, 8)),
    ("channel", 1, 0.95, (2, 16, 3, 8, 8)),
    ("head", 1, 1.95, (2, 12, 2, 8, 8)),
    ("channel", 1, 1.95, (2, 12, 2, 8, 8)),
    ("head", 1, 0.95, (2, 13, 2, 8, 16)),
    ("channel", 1, 0.95, (2, 16, 2, 16, 8)),
    ("head", 2, 1.95, (2, 7, 2, 8, 8)),
    ("channel", 3, 0.95, (1, 5, 2, 4, 6)),
])
def test_backward_oracle_matches_autograd(gates, u, beta_max, dims):
    b, t, h, dk, dv = dims
    rng = np.random.default_rng(zlib.crc32(repr((gates, u, beta_max, dims)).encode()))
    x = make(rng, b, t, h, dk, dv, u, gates, beta_max)
    dy = rng.standard_normal((b, t, h, dv))
    dsf = rng.standard_normal((b, h, dk, dv))
    scale = 1 / np.sqrt(dk)
    tt = {n: None if a is None else torch.tensor(a, dtype=torch.float64, requires_grad=True) for n, a in x.items()}
    y, S = forward_torch(tt["q"], tt["k"], tt["v"], tt["e"], tt["w"], tt["g"], tt["s0"], scale, u)
    loss = (y * torch.tensor(dy)).sum() + (S * torch.tensor(dsf)).sum()
    loss.backward()
    got = oracle.recurrent_backward(x["q"], x["k"], x["v"], x["e"], x["w"], x["g"], x["s0"], dy, dsf, scale, u)
    # the forward used by the oracle is the oracle's own recurrence
    y0, s0 = oracle.householder("recurrent", x["q"], x["k"], x["v"], x["e"], x["w"], x["g"], x["s0"], u,
                                scale=scale)
    assert np.abs(y.detach().numpy() - y0).max() < 1e-12 and np.abs(S.detach().numpy() - s0).max() < 1e-12
    pairs = dict(d_q="q", d_k="k", d_v="v", d_erase="e", d_write="w", d_g="g", d_state="s0")
    for gk, xk in pairs.items():
        if tt[xk] is None:
            assert got[gk] is None
            continue
        ref = tt[xk].grad.numpy()
        assert got[gk].shape == ref.shape, (gk, got[gk].shape, ref.shape)
        assert np.abs(got[gk] - ref).max() < 1e-10, (gk, np.abs(got[gk] - ref).max())

"""Parity at BASELINE's full sizes, through properties that hold at any size.

The CPU oracle covers small sizes (the other GPU tests); at the benchmark
shapes it would take hours, so the tensor-core paths are checked against
independent evidence on the GPU:
  * against DeltaPath::Recurrent: the sequence walked token by token by the
    fp32 decode tick (a different kernel and a different algorithm), within
    the bf16 bound of 2e-2 max-abs on y and on the final state;
  * a sequence cut at a chunk boundary and run as two calls (the state carried
    between them) gives bit-identical results to one call
    (src/delta/tests.rs:465-494);
  * a batch subset gives bit-identical rows (heads are independent,
    src/delta/recurrent.rs:41-99), which is what the batch x head sharding
    relies on.
Inputs follow the benchmark recipes (bench.make_prefill), seeded."""
import importlib
import math

import pytest
import torch

import bench

pytestmark = pytest.mark.gpu
dn = importlib.import_module("burn-deltanet_b200")
abi = importlib.import_module("burn-deltanet_b200._abi")

TOL = 2e-2  # bf16 q/k/v, fp32 state and accumulation


def run(x, u, recurrent=False, sl=slice(None), t0=0, t1=None, state=None):
    q, k, v, e, w, g = (x[n] for n in ("q", "k", "v", "erase", "write", "g"))
    t1 = q.shape[1] if t1 is None else t1
    rows = lambda t, per: t[sl, t0 * per:t1 * per].contiguous()
    gated = g is not None
    return dn.delta_chunk_recalculated(
        rows(q, 1), rows(k, u), rows(v, u), rows(e, u), rows(w, u), rows(g, 1) if gated else None,
        (x["state"][sl] if state is None else state).contiguous(), gated, 64, 1.0 / math.sqrt(128),
        n_householder=u, out_dtype=torch.float32, recurrent=recurrent)


@pytest.mark.parametrize("kind,batch,tokens,u", [
    ("deltanet", 8, 4096, 1),       # config 2
    ("deltaproduct", 4, 8192, 2),   # config 4, u = 2
    ("deltaproduct", 4, 8192, 3),   # config 4, u = 3
    ("gdn2", 16, 16384, 1),         # config 5 (one GPU's view of the whole batch)
])
def test_full_size_properties(kind, batch, tokens, u):
    x = bench.make_prefill(kind, batch, tokens, u, "cuda", 11)
    assert abi.lib().dc_device_status(1) == 0
    y, s = run(x, u)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all() and torch.isfinite(s).all()

    # against the token-by-token recurrence
    y_r, s_r = run(x, u, recurrent=True)
    torch.cuda.synchronize()
    ey, es = (y - y_r).abs().max().item(), (s - s_r).abs().max().item()
    print(f"{kind} B={batch} T={tokens} u={u}: max |y - y_rec| {ey:.3e}, max |S - S_rec| {es:.3e}")
    assert ey < TOL and es < TOL, (ey, es)
    del y_r, s_r

    # two calls cut at a chunk boundary, the state carried between them
    step = 64 // math.gcd(64, u)  # tokens whose u micro-steps fill whole 64-row chunks
    cut = (tokens // 2) // step * step
    y1, s1 = run(x, u, t1=cut)
    y2, s2 = run(x, u, t0=cut, state=s1)
    torch.cuda.synchronize()
    assert torch.equal(torch.cat([y1, y2], dim=1), y) and torch.equal(s2, s)
    del y1, y2, s1, s2

    # a batch subset: the same rows, bit for bit
    sub = slice(1, 3)
    y_b, s_b = run(x, u, sl=sub)
    torch.cuda.synchronize()
    assert torch.equal(y_b, y[sub]) and torch.equal(s_b, s[sub])
    assert abi.lib().dc_device_status(1) == 0

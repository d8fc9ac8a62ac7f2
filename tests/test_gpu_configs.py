"""GPU parity at the BASELINE configurations' own shapes and recipes.

Config 1 is the reference's CPU-runnable case: the Gated DeltaNet core in
float32, B=2 T=512 H=4 dk=dv=64, chunk 64, q and k L2-normalised N(0,1),
v ~ N(0,1), beta = sigmoid(N(0,1)), log alpha = -exp(a_h) softplus(x) with
a_h ~ U(0, ln 16) per head, S0 = 0, seed 0.  Its check is the reference's:
the chunkwise forward and the recurrent step() path agree on y and on the
final state (src/delta/tests.rs:300-363).  Here both GPU paths are also held
to the float64 oracle (the reference algorithm restated in C, pinned to the
reference's golden vectors), at the north star's 1e-4 relative for the fp32
path: max |gpu - oracle| <= 1e-4 * max(1, max |oracle|).

Config 3's recipe (Gated DeltaNet decode from S0 ~ N(0, 0.02^2)) is checked
over 1024 ticks in test_gpu_core.py; configs 2, 4 and 5 at full size in
test_gpu_fullsize.py."""
import importlib

import numpy as np
import pytest
import torch

import oracle
from _inputs import config_inputs

pytestmark = pytest.mark.gpu
dn = importlib.import_module("burn-deltanet_b200")
abi = importlib.import_module("burn-deltanet_b200._abi")

F32_TOL = 1e-4  # the north star's bound for the fp32 path


def _dev(x):
    return None if x is None else torch.from_numpy(np.ascontiguousarray(x)).to("cuda", torch.float32)


def _rel(got, want):
    return np.abs(got.double().cpu().numpy() - want).max() / max(1.0, np.abs(want).max())


def test_config1_chunk_equals_recurrent_equals_oracle():
    raw = config_inputs(1, np.random.default_rng(0), 2, 512, 4, 64, 64)
    assert raw["g"].shape == (2, 512, 4, 1) and raw["erase"].shape == (2, 512, 4, 1)
    ins = [_dev(raw[n]) for n in ("q", "k", "v", "erase", "write", "g", "state")]
    inp = dn.DeltaInput(*ins)
    assert abi.lib().dc_device_status(1) == 0
    y_c, s_c = inp.run(dn.DeltaPath.ChunkRecalculated(64))
    y_r, s_r = inp.run(dn.DeltaPath.Recurrent())
    torch.cuda.synchronize()
    assert y_c.dtype == torch.float32 and tuple(y_c.shape) == (2, 512, 4, 64)
    y_o, s_o = oracle.householder("recurrent", raw["q"], raw["k"], raw["v"], raw["erase"], raw["write"], raw["g"],
                                  raw["state"], 1)
    errs = {"chunk y": _rel(y_c, y_o), "chunk S": _rel(s_c, s_o), "recurrent y": _rel(y_r, y_o),
            "recurrent S": _rel(s_r, s_o)}
    # the reference's own check: chunkwise == recurrent
    errs["chunk vs recurrent y"] = _rel(y_c, y_r.double().cpu().numpy())
    errs["chunk vs recurrent S"] = _rel(s_c, s_r.double().cpu().numpy())
    print("config 1: " + ", ".join(f"{k} {v:.2e}" for k, v in errs.items()))
    for name, e in errs.items():
        assert e <= F32_TOL, (name, e)
    # the oracle's own chunk path (the reference's chunkwise arithmetic) agrees as well
    y_oc, s_oc = oracle.householder("chunk", raw["q"], raw["k"], raw["v"], raw["erase"], raw["write"], raw["g"],
                                    raw["state"], 1, chunk_len=64)
    assert np.abs(y_oc - y_o).max() < 1e-9 and np.abs(s_oc - s_o).max() < 1e-9
    assert abi.lib().dc_device_status(1) == 0


def test_config1_split_calls_equal_one_call():
    """src/delta/tests.rs:465-494 at config 1's shapes: two calls cut at a chunk boundary, the state carried
    between them, give the one call's y and final state."""
    raw = config_inputs(1, np.random.default_rng(0), 2, 512, 4, 64, 64)
    t = {n: _dev(raw[n]) for n in ("q", "k", "v", "erase", "write", "g", "state")}

    def call(t0, t1, state):
        sl = lambda x: x[:, t0:t1].contiguous()
        return dn.delta_chunk_recalculated(sl(t["q"]), sl(t["k"]), sl(t["v"]), sl(t["erase"]), sl(t["write"]),
                                           sl(t["g"]), state, True, 64, 1.0 / 8.0)

    y, s = call(0, 512, t["state"])
    y1, s1 = call(0, 192, t["state"])
    y2, s2 = call(192, 512, s1)
    torch.cuda.synchronize()
    assert torch.equal(torch.cat([y1, y2], 1), y) and torch.equal(s2, s)

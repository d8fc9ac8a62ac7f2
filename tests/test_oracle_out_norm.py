"""The output-norm oracle (oracle/out_norm.py) against independent implementations.

The plain form against torch.nn.functional.rms_norm (PyTorch's RMSNorm: x / sqrt(mean(x^2) + eps) * w);
the gated form against torch's silu on top of it; a zero row stays zero (the epsilon guard)."""
import numpy as np
import torch

import oracle


def test_plain_form_matches_torch_rms_norm():
    rng = np.random.default_rng(3)
    y = rng.standard_normal((2, 5, 3, 40)) * 3.0
    w = rng.uniform(0.5, 1.5, 40)
    got = oracle.out_norm(y, None, w, 1e-5)
    ref = torch.nn.functional.rms_norm(torch.from_numpy(y), (40,), torch.from_numpy(w), 1e-5).numpy()
    assert np.abs(got - ref).max() < 1e-12


def test_gated_form_is_the_plain_form_times_silu_of_the_gate():
    rng = np.random.default_rng(4)
    y, gate = rng.standard_normal((3, 7, 2, 16)), rng.standard_normal((3, 7, 2, 16)) * 4.0
    w = rng.uniform(0.5, 1.5, 16)
    got = oracle.out_norm(y, gate, w, 1e-6)
    plain = torch.nn.functional.rms_norm(torch.from_numpy(y), (16,), torch.from_numpy(w), 1e-6)
    ref = (plain * torch.nn.functional.silu(torch.from_numpy(gate))).numpy()
    assert np.abs(got - ref).max() < 1e-12


def test_zero_rows_stay_zero():
    y = np.zeros((1, 2, 1, 8))
    assert np.array_equal(oracle.out_norm(y, np.ones_like(y), np.ones(8), 1e-5), y)

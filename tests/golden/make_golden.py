"""Extract the reference's float64 golden vectors into a JSON fixture.

The reference pins its delta-rule core to flash-linear-attention's naive
recurrences with one fixed input (``src/delta/tests/reference.rs:17-59``,
written by ``scripts/gen_fixture.py`` at seed 20260826, dims
``[batch, seq, heads, dk, dv] = [2, 9, 2, 4, 6]``).  Those vectors are data,
not code: this script reads them out of ``reference.rs`` as text and writes
``fla_naive_b2_t9_h2_k4_v6.json`` beside itself, which the tests load.

Run it where the reference checkout is present::

    python tests/golden/make_golden.py /path/to/burn-deltanet

The GPU box never runs it; it uses the committed JSON.
"""
from __future__ import annotations

import json
import os
import re
import sys

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "fla_naive_b2_t9_h2_k4_v6.json")

# name in reference.rs -> (key in the fixture, shape builder from DIMS)
FIELDS = {
    "IN_Q": ("q", lambda b, t, h, k, v: [b, t, h, k]),
    "IN_K": ("k", lambda b, t, h, k, v: [b, t, h, k]),
    "IN_V": ("v", lambda b, t, h, k, v: [b, t, h, v]),
    "IN_BETA": ("beta", lambda b, t, h, k, v: [b, t, h]),
    "IN_G": ("g", lambda b, t, h, k, v: [b, t, h]),
    "IN_STATE": ("state", lambda b, t, h, k, v: [b, h, k, v]),
    "IN_B": ("b", lambda b, t, h, k, v: [b, t, h, k]),
    "IN_W": ("w", lambda b, t, h, k, v: [b, t, h, v]),
    "IN_GK": ("gk", lambda b, t, h, k, v: [b, t, h, k]),
    "UNGATED_Y": ("ungated_y", lambda b, t, h, k, v: [b, t, h, v]),
    "UNGATED_STATE": ("ungated_state", lambda b, t, h, k, v: [b, h, k, v]),
    "GATED_Y": ("gated_y", lambda b, t, h, k, v: [b, t, h, v]),
    "GATED_STATE": ("gated_state", lambda b, t, h, k, v: [b, h, k, v]),
    "GDN2_Y": ("gdn2_y", lambda b, t, h, k, v: [b, t, h, v]),
    "GDN2_STATE": ("gdn2_state", lambda b, t, h, k, v: [b, h, k, v]),
}


def main(reference_root: str) -> None:
    path = os.path.join(reference_root, "src", "delta", "tests", "reference.rs")
    text = open(path).read()
    dims = [int(x) for x in re.search(r"pub const DIMS: \[usize; 5\] = \[([^\]]*)\]", text).group(1).split(",")]
    fixture = {
        "source": "burn-deltanet src/delta/tests/reference.rs:17-59 (flash-linear-attention naive "
                  "recurrences at float64, scripts/gen_fixture.py, seed 20260826)",
        "dims": dims,
        "tensors": {},
    }
    for name, (key, shape_of) in FIELDS.items():
        m = re.search(rf"pub const {name}: &\[f64\] = &\[([^\]]*)\];", text)
        values = [float(x) for x in m.group(1).split(",") if x.strip()]
        shape = shape_of(*dims)
        n = 1
        for s in shape:
            n *= s
        assert len(values) == n, (name, len(values), shape)
        fixture["tensors"][key] = {"shape": shape, "data": values}
    with open(OUT, "w") as f:
        json.dump(fixture, f)
    print("wrote", OUT)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to the burn-deltanet checkout>")
    main(sys.argv[1])

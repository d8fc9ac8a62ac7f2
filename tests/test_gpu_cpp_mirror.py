"""The C++ host mirror (burn-deltanet_b200/csrc/delta_core.hpp) on the GPU:
tests/cpp/host_mirror_test runs DeltaInput::run (chunk and recurrent paths),
delta_step and the sanity exceptions against the linked CPU oracle."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "tests", "cpp", "host_mirror_test")


def ensure_built():
    if not os.path.exists(BIN):
        subprocess.run(["sh", os.path.join(ROOT, "tests", "cpp", "build.sh")], check=True)


def test_cpp_mirror_builds():
    ensure_built()
    assert os.access(BIN, os.X_OK)


@pytest.mark.gpu
def test_cpp_mirror_on_gpu():
    ensure_built()
    r = subprocess.run([BIN], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr

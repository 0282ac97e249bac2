"""The reference's OWN GPU gate (tests/unit/test_cuda.c), compiled from its
sources and linked against libdsv4_b200.so in place of the reference's
build/dsv4_cuda.o (oracle/Makefile target `refgate`). Passing it is the
drop-in claim: the unchanged reference host code talks to this backend.
The binary is built where the reference checkout exists and travels as a
built file; without it the test is skipped."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GATE = os.path.join(REPO, "oracle", "_ref", "test_cuda_b200")


@pytest.mark.skipif(not os.path.exists(GATE), reason="reference gate not built here")
def test_reference_cuda_gate_passes_on_this_backend():
    r = subprocess.run([GATE], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "CUDA GATE PASSED" in r.stdout

"""Shared test set-up.

Markers: ``gpu`` marks every test that needs a B200 (run with ``-m gpu``);
everything else runs on CPU (``-m "not gpu"``).
"""
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "deepseek-v4-in-c_b200")
for p in (os.path.join(REPO, "oracle"), PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (CUDA device)")


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(REPO, "tests", "golden", "golden.npz"))


@pytest.fixture(scope="session")
def flash_sample():
    """The benchmark's CPU-baseline sample (three Flash layers, all 256
    experts, the 129280-token head) as host weights, built once per session
    (minutes of host work)."""
    import dsv4_model as M
    return M.SyntheticModel(M.flash_sample_config(), seed=0, fast=True)


@pytest.fixture(scope="session")
def port():
    import oracle
    return oracle.Checker("port")


def vrel(got, ref):
    """Vector-scaled relative error, the reference GPU gate's metric
    (tests/unit/test_cuda.c:159-170): |got-ref| / max(rms(ref), |got|, |ref|)."""
    got = np.asarray(got, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    rms = np.sqrt(np.mean(ref * ref)) if ref.size else 0.0
    den = np.maximum(rms, np.maximum(np.abs(got), np.abs(ref)))
    with np.errstate(invalid="ignore", divide="ignore"):
        r = np.where(den > 0, np.abs(got - ref) / den, 0.0)
    return float(r.max()) if r.size else 0.0

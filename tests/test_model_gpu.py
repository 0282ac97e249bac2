"""Whole-token decode on the B200: the tiny synthetic
model, a 32-token prompt and 64 greedy tokens must give the SAME argmax at
every position as the reference's own layer code (golden from
dsv4_layer_forward, tests/golden/make_c4_golden.py); logits agree to within
the model-level tolerance the reference's own model oracle uses (2e-3,
tests/unit/test_model_oracle.c:266-283)."""
import os

import numpy as np
import pytest

import dsv4_b200 as B
import dsv4_model as M
from conftest import vrel

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def tiny():
    B.init()
    g = np.load(os.path.join(REPO, "tests", "golden", "c4_golden.npz"))
    sm = M.SyntheticModel(M.tiny_config(), seed=0)
    m = B.Model(sm, 256)
    yield g, sm, m
    m.close()


def test_config4_greedy_tokens_identical(tiny):
    g, sm, m = tiny
    out = m.generate(g["prompt"], 64)
    assert list(out) == list(g["tokens"])


def test_config4_logits_stepwise(tiny):
    g, sm, m = tiny
    m.begin(g["prompt"])
    rows, toks = [], []
    for pos in range(32 + 64):
        t, lg = m.step(want_logits=True)
        if pos + 1 >= 32:
            rows.append(lg)
            toks.append(t)
    assert toks == list(g["tokens"])
    rows = np.stack(rows)
    for i in range(8):
        assert vrel(rows[i], g["logits_head"][i]) < 2e-3
    for i in range(2):
        assert vrel(rows[-2 + i], g["logits_tail"][i]) < 2e-3
    # every decision had more room than the logits moved
    dev = np.abs(rows[:8] - g["logits_head"]).max(axis=1)
    assert np.all(dev < g["margin"][:8])


def test_config4_restart_is_reproducible(tiny):
    g, sm, m = tiny
    a = m.generate(g["prompt"], 16)
    b = m.generate(g["prompt"], 16)
    assert list(a) == list(b) == list(g["tokens"][:17])

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


def test_flash_geometry_slice_against_oracle():
    """Config-5 shapes (hidden 4096, 64 heads x 512, indexer 64 x 128, FP4
    experts 2048 x 4096) on two layers (CSA ratio 4 and HCA ratio 128) and 16
    experts, with index_topk lowered to 4 so selection runs within the 24
    positions: argmax identical to the oracle at every position."""
    import oracle as O
    B.init()
    d = M.flash_slice(n_layers=2, n_experts=16, ratios=(4, 128))
    d["index_topk"] = 4
    sm = M.SyntheticModel(d, seed=3)
    m = B.Model(sm, 64)
    prompt = np.random.default_rng(1).integers(0, d["vocab"], 8).astype(np.int32)
    out = m.generate(prompt, 16)
    ref, lg = O.model_greedy_port(sm, prompt, 16, 64, keep_logits=True)
    assert list(out) == list(ref)
    m.begin(prompt)
    for pos in range(8):
        t, row = m.step(want_logits=True)
    assert vrel(row, lg[0]) < 2e-3
    m.close()


def test_synthetic_on_device_model_runs():
    """The on-device generator (config 5's path) on the tiny geometry: runs,
    is deterministic in its seed, and the host-driven decode entry agrees
    with graph-driven generation."""
    B.init()
    co = M.ConfigOnly(M.tiny_config())
    a = B.Model(co, 128, synthetic_seed=7)
    prompt = np.arange(5, dtype=np.int32)
    ga = a.generate(prompt, 10)
    b = B.Model(co, 128, synthetic_seed=7)
    assert list(b.generate(prompt, 10)) == list(ga)
    b.begin(prompt)
    toks = list(prompt)
    outs = []
    for pos in range(5 + 10):
        nxt = b.decode(toks[pos], pos)
        if pos >= 4:
            outs.append(nxt)
            if pos + 1 >= len(toks):
                toks.append(nxt)
    assert outs == list(ga)
    a.close()
    b.close()


def test_flash_sample_against_reference(flash_sample):
    """The benchmark's CPU-baseline sample -- three Flash-geometry layers
    (compress ratios 0 / 4 / 128), all 256 FP4 experts, the 129280-token
    head -- decoded on the GPU from a 16-token prompt for 16 greedy tokens:
    the argmax at every position is the reference's own dsv4_layer_forward
    token loop's (oracle/_ref, the CLI loop of src/cli/dsv4_run.c:444-483)."""
    import oracle as O
    assert os.path.exists(O.REF_SO), "oracle/_ref/libdsv4ref.so is built with the package"
    B.init()
    sm = flash_sample
    prompt = np.random.default_rng(11).integers(0, sm.d["vocab"], 16).astype(np.int32)
    m = B.Model(sm, 64)
    out = m.generate(prompt, 16)
    m.close()
    ref, _ = O.model_greedy_ref(sm, prompt, 16, 64)
    assert len(ref) == 17
    assert list(out) == list(ref)

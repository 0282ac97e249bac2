"""Batched prefill on the device (dsv4b_model_prefill / _generate_prefill,
the reference's --batch prompt path: src/cli/dsv4_run.c:391-442 over
dsv4_layer_forward_n, src/model/dsv4_layer.c:856-918). Every token's
arithmetic is that of a decode step, so the tokens must be the per-token
path's bit for bit: the config-4 golden tokens at pass sizes that leave a
ragged last pass and that wrap the 16-position window ring inside a pass;
the logits of the first step after the prompt equal the per-token model's;
a 100-token prompt against the reference's own batched prompt path
(oracle/_ref); a Flash slice (FP4 experts, the tensor-core expert union)
against its per-token model; and the benchmark's Flash sample (all 256
experts, the full head) against the reference's batched prompt path."""
import os

import numpy as np
import pytest

import dsv4_b200 as B
import dsv4_model as M

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_config4_prefill_matches_golden():
    B.init()
    g = np.load(os.path.join(REPO, "tests", "golden", "c4_golden.npz"))
    sm = M.SyntheticModel(M.tiny_config(), seed=0)
    m = B.Model(sm, 256)
    # three calls per pass size: a pass shape runs eagerly the first time,
    # is captured as a graph the second and replayed the third
    for chunk in (1, 2, 5, 16, 17, 32, 64):
        for rep in range(3):
            out = m.generate_prefill(g["prompt"], 64, chunk)
            assert list(out) == list(g["tokens"]), "chunk %d, call %d" % (chunk, rep)
        assert B.lib().dsv4b_model_prefill_kernels(m.h) > 0
    # the state a prefill leaves: the next step is the per-token path's, its
    # logits bit for bit
    prompt = g["prompt"]
    m.begin(prompt)
    for _ in range(len(prompt)):
        first, _ = m.step()
    want_tok, want_lg = m.step(want_logits=True)
    assert m.prefill(prompt, 7) == first
    tok, lg = m.step(want_logits=True)
    assert tok == want_tok and lg.tobytes() == want_lg.tobytes()
    # pass sizes out of range are refused
    for chunk in (0, 65):
        assert B.lib().dsv4b_model_prefill(m.h, prompt.ctypes.data, len(prompt), chunk) == -1
    m.close()
    # a batched model has no prefill
    mb = B.Model(sm, 64, n_seq=2)
    assert B.lib().dsv4b_model_prefill(mb.h, prompt.ctypes.data, len(prompt), 8) == -1
    mb.close()


def test_config4_long_prompt_against_reference_prefill():
    import oracle as O
    assert os.path.exists(O.REF_SO), "oracle/_ref/libdsv4ref.so is built with the package"
    B.init()
    sm = M.SyntheticModel(M.tiny_config(), seed=0)
    prompt = np.random.default_rng(21).integers(0, sm.d["vocab"], 100).astype(np.int32)
    ref, _ = O.model_prefill_ref(sm, prompt, 20, 160, 32)
    m = B.Model(sm, 160)
    assert list(m.generate_prefill(prompt, 20, 32)) == list(ref)
    assert list(m.generate(prompt, 20)) == list(ref)
    m.close()


def test_flash_slice_prefill_matches_per_token():
    """Config-5 shapes generated on the device (CSA, HCA and window layers,
    16 FP4 experts on the tensor-core union path)."""
    B.init()
    co = M.ConfigOnly(M.flash_slice(n_layers=3, n_experts=16, ratios=(4, 128)))
    prompt = np.random.default_rng(9).integers(0, co.d["vocab"], 70).astype(np.int32)
    m = B.Model(co, 160, synthetic_seed=5)
    want = m.generate(prompt, 12)
    for chunk in (32, 64):
        for rep in range(3):
            assert list(m.generate_prefill(prompt, 12, chunk)) == list(want), "chunk %d, call %d" % (chunk, rep)
    m.close()


def test_flash_sample_prefill_against_reference(flash_sample):
    """The benchmark's CPU-baseline sample (three Flash layers, all 256
    experts, the 129280-token head): a 40-token prompt in passes of 32 and 8
    against the reference's own batched prompt path."""
    import oracle as O
    B.init()
    sm = flash_sample
    prompt = np.random.default_rng(13).integers(0, sm.d["vocab"], 40).astype(np.int32)
    ref, _ = O.model_prefill_ref(sm, prompt, 8, 64, 32)
    m = B.Model(sm, 64)
    assert list(m.generate_prefill(prompt, 8, 32)) == list(ref)
    m.close()

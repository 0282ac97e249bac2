"""Batched decode: n_seq sequences stepped in lockstep by one graph, every
launch covering all of them. Each sequence's arithmetic is that of a
one-sequence model (a grid dimension, or one GEMV item per sequence), so
its greedy tokens must be exactly the ones the one-sequence model gives for
its prompt, and the reference's where that is pinned: the config-4 golden
prompt (tokens of the reference's dsv4_layer_forward loop,
tests/golden/make_c4_golden.py) and the benchmark's three-layer Flash sample
against oracle/_ref."""
import os

import numpy as np
import pytest

import dsv4_b200 as B
import dsv4_model as M

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _prompts(first, n_seq, vocab, seed):
    rng = np.random.default_rng(seed)
    rows = [np.asarray(first, np.int32)]
    for _ in range(n_seq - 1):
        rows.append(rng.integers(0, vocab, len(first)).astype(np.int32))
    return np.stack(rows)


def test_config4_batch_matches_reference_and_single():
    B.init()
    g = np.load(os.path.join(REPO, "tests", "golden", "c4_golden.npz"))
    sm = M.SyntheticModel(M.tiny_config(), seed=0)
    prompts = _prompts(g["prompt"], 4, sm.d["vocab"], 3)
    mb = B.Model(sm, 256, n_seq=4)
    assert B.lib().dsv4b_model_n_seq(mb.h) == 4
    out = mb.generate_batch(prompts, 64)
    # the one-sequence calls refuse a batched model
    assert B.lib().dsv4_cuda_model_generate(mb.h, prompts[0].ctypes.data, prompts.shape[1], 4,
                                            np.zeros(8, np.int32).ctypes.data) == -1
    again = mb.generate_batch(prompts, 64)
    mb.close()
    assert list(out[0]) == list(g["tokens"])
    assert np.array_equal(out, again)
    m1 = B.Model(sm, 256)
    for b in range(1, 4):
        assert list(out[b]) == list(m1.generate(prompts[b], 64)), "sequence %d" % b
    m1.close()


def test_flash_slice_batch8_matches_single():
    """Config-5 shapes (CSA and HCA layers and a window layer, 16 FP4
    experts) generated on the device, 8 sequences against the one-sequence
    model of the same seed, through the graph-driven and the host-driven
    entry points."""
    B.init()
    co = M.ConfigOnly(M.flash_slice(n_layers=3, n_experts=16, ratios=(4, 128)))
    prompts = _prompts(np.arange(12, dtype=np.int32) * 7, 8, co.d["vocab"], 5)
    mb = B.Model(co, 96, synthetic_seed=5, n_seq=8)
    out = mb.generate_batch(prompts, 12)
    # the host-driven entry: every sequence's token in, the next ones out
    mb.begin_batch(prompts)
    toks = [prompts[:, p] for p in range(prompts.shape[1])]
    host = []
    for pos in range(prompts.shape[1] + 12):
        nxt = mb.decode_batch(toks[pos], pos)
        if pos + 1 >= prompts.shape[1]:
            host.append(nxt)
            if pos + 1 >= len(toks):
                toks.append(nxt)
    mb.close()
    assert np.array_equal(np.stack(host, axis=1), out)
    m1 = B.Model(co, 96, synthetic_seed=5)
    for b in range(8):
        assert list(out[b]) == list(m1.generate(prompts[b], 12)), "sequence %d" % b
    m1.close()


def test_flash_sample_batch_against_reference(flash_sample):
    """The benchmark's CPU-baseline sample (three Flash layers, all 256
    experts, the 129280-token head), three sequences: sequence 0 is the
    reference's token loop's (oracle/_ref) for its prompt, the others the
    one-sequence model's."""
    import oracle as O
    assert os.path.exists(O.REF_SO), "oracle/_ref/libdsv4ref.so is built with the package"
    B.init()
    sm = flash_sample
    first = np.random.default_rng(11).integers(0, sm.d["vocab"], 16).astype(np.int32)
    prompts = _prompts(first, 3, sm.d["vocab"], 12)
    mb = B.Model(sm, 64, n_seq=3)
    out = mb.generate_batch(prompts, 16)
    mb.close()
    ref, _ = O.model_greedy_ref(sm, prompts[0], 16, 64)
    assert list(out[0]) == list(ref)
    m1 = B.Model(sm, 64)
    for b in range(1, 3):
        assert list(out[b]) == list(m1.generate(prompts[b], 16)), "sequence %d" % b
    m1.close()

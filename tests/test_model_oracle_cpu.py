"""The oracle's restated whole-token decode (oracle/dsv4_oracle_model.c) must
reproduce the REFERENCE's greedy decode of BASELINE config 4 exactly: every
token, and the logits bit for bit (golden from the reference's own
dsv4_layer_forward: tests/golden/make_c4_golden.py). CPU only."""
import os

import numpy as np

import dsv4_model as M
import oracle as O

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_tiny_model_port_matches_reference_golden():
    g = np.load(os.path.join(REPO, "tests", "golden", "c4_golden.npz"))
    sm = M.SyntheticModel(M.tiny_config(), seed=0)
    out, lg = O.model_greedy_port(sm, g["prompt"], 64, 256)
    assert list(out) == list(g["tokens"])
    assert lg[:8].tobytes() == g["logits_head"].tobytes()
    assert lg[-2:].tobytes() == g["logits_tail"].tobytes()

"""A checkpoint bound to HBM: the config-4 weights written as .safetensors in
the released layout (tests/ckpt_writer.py), bound by the REFERENCE's own
reader and binder (oracle/_ref), handed to dsv4_cuda_model_create, and
decoded on the device: the greedy tokens are the reference's golden tokens
for the golden prompt (tests/golden/make_c4_golden.py)."""
import os

import numpy as np
import pytest

import dsv4_b200 as B
import dsv4_model as M

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_bound_checkpoint_decodes_golden_tokens(tmp_path):
    import oracle as O
    import ckpt_writer as W
    assert os.path.exists(O.REF_SO), "oracle/_ref/libdsv4ref.so is built with the package"
    B.init()
    g = np.load(os.path.join(REPO, "tests", "golden", "c4_golden.npz"))
    sm = M.SyntheticModel(M.tiny_config(), seed=0)
    W.write_checkpoint(sm, str(tmp_path))
    bound = O.BoundCheckpoint(str(tmp_path), sm)
    m = B.Model(bound, 256)
    out = m.generate(g["prompt"], 64)
    m.close()
    bound.close()
    assert list(out) == list(g["tokens"])

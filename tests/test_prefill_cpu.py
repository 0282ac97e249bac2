"""The reference's batched prompt path (oracle/_ref: dsv4_layer_forward_n in
passes, src/cli/dsv4_run.c:391-442) gives the config-4 golden tokens (its
per-token loop's, tests/golden/make_c4_golden.py) at every pass size, ragged
last passes and a 16-position window ring that wraps inside one pass
included: the pin the device prefill (tests/test_prefill_gpu.py) is held
to. CPU only."""
import os

import numpy as np
import pytest

import dsv4_model as M

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.skipif(not os.path.exists(os.path.join(REPO, "oracle", "_ref", "libdsv4ref.so")),
                                reason="oracle/_ref is built from the reference's sources (make -C oracle ref)")


@pytest.mark.parametrize("chunk", [1, 2, 5, 16, 32, 64])
def test_reference_prefill_matches_golden(chunk):
    import oracle as O
    g = np.load(os.path.join(REPO, "tests", "golden", "c4_golden.npz"))
    sm = M.SyntheticModel(M.tiny_config(), seed=0)
    out, tp = O.model_prefill_ref(sm, g["prompt"], 24, 64, chunk)
    assert list(out) == list(g["tokens"][:25])
    assert tp.shape == (-(-len(g["prompt"]) // chunk), sm.d["n_layers"]) and (tp > 0).all()


def test_reference_prefill_refuses_bad_chunk():
    import oracle as O
    sm = M.SyntheticModel(M.tiny_config(), seed=0)
    with pytest.raises(RuntimeError):
        O.model_prefill_ref(sm, np.arange(8), 2, 16, 65)

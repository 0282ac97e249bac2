"""The checkpoint path: a directory of .safetensors in the released layout
(tests/ckpt_writer.py, written from the config-4 synthetic model) is bound by
the REFERENCE's own reader and binder (oracle/_ref: src/io/dsv4_st.c,
src/model/dsv4_bind.c, experts by the names of src/cache/dsv4_cache.c), and
every tensor the binder and the expert reads hand over is byte-identical to
the synthetic model's. tests/test_checkpoint_gpu.py then builds the device
model from those structs."""
import os

import numpy as np
import pytest

import dsv4_model as M

pytestmark = pytest.mark.skipif(
    not os.path.exists(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "oracle", "_ref", "libdsv4ref.so")),
    reason="oracle/_ref is built from the reference's sources (make -C oracle ref)")


def test_reference_binder_roundtrip(tmp_path):
    import oracle as O
    import ckpt_writer as W
    sm = M.SyntheticModel(M.tiny_config(), seed=0)
    tl = W.write_checkpoint(sm, str(tmp_path))
    bound = O.BoundCheckpoint(str(tmp_path), sm)
    ne = sm.d["n_experts"]
    for name, dt, shp, path in tl:
        n = W.nbytes(dt, shp)
        got = W.data((bound.mw, bound.layers, bound.experts), path, ne, n)
        want = W.data((sm.mw, sm.layers, sm.experts), path, ne, n)
        assert got is not None, name                # the binder hands over every tensor
        if want is not None:
            assert np.array_equal(got, want), name
    # the structs' shapes and formats as the reference binds them
    for L in range(sm.d["n_layers"]):
        a, b = bound.layers[L].attn.wq_b, sm.layers[L].attn.wq_b
        assert (a.wdt, a.rows, a.cols, a.blk_r, a.blk_c) == (b.wdt, b.rows, b.cols, b.blk_r, b.blk_c)
        assert bound.layers[L].has_idx == sm.layers[L].has_idx
    assert bound.mw.wdt == sm.mw.wdt
    bound.close()

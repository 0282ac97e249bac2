"""Golden vectors for the config-2 router from the reference's own PyTorch
restatement of the checkpoint model (tools/dsv4_ref.py of the reference
checkout): fp32 router logits, SIGMOID scores, top-6 selection with an
optional selection-only bias, weights renormalised to sum 1 and scaled.

The reference's C implements only sqrt(softplus) scoring
(src/core/dsv4_ops.c:102-141), so this is the reference-held source that
pins the sigmoid path of the oracle's restated router (dsv4o_route) and its
fp32 router GEMV. Inputs are regenerated from the seed by the test (the
router matrix is 4 MB); a checksum of their bytes is stored beside the
outputs.

    python tests/golden/make_route_golden.py [REF_DIR]

Needs the reference checkout (argument, REF_DIR, else `reference` beside the
repository) and torch; writes tests/golden/route_golden.npz.
"""
import hashlib
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "route_golden.npz")
SEED, HIDDEN, N_EXPERTS, TOPK, TRIALS = 2026, 4096, 256, 6, 6


def inputs():
    """Config 2's router: W ~ N(0, 0.02) fp32 [256][4096]; per trial x ~ N(0, 1)
    and (odd trials) a selection bias ~ N(0, 0.05)."""
    rng = np.random.default_rng(SEED)
    W = rng.standard_normal((N_EXPERTS, HIDDEN), dtype=np.float32) * np.float32(0.02)
    xs = rng.standard_normal((TRIALS, HIDDEN), dtype=np.float32)
    bias = (rng.standard_normal((TRIALS, N_EXPERTS)) * 0.05).astype(np.float32)
    bias[0::2] = 0.0
    return W, xs, bias


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def main():
    ref_dir = (sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REF_DIR")
               or os.path.join(os.path.dirname(REPO), "reference"))
    spec = importlib.util.spec_from_file_location("dsv4_ref", os.path.join(ref_dir, "tools", "dsv4_ref.py"))
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    import torch
    W, xs, bias = inputs()
    tw = torch.from_numpy(W)
    logits, scores, idx, wts = [], [], [], []
    for t in range(TRIALS):
        lg = torch.nn.functional.linear(torch.from_numpy(xs[t])[None], tw)      # fp32 router
        b = torch.from_numpy(bias[t]) if t % 2 else None
        w, i = ref.route(lg, b, None, None, TOPK, 1.0, score_func="sigmoid")
        logits.append(lg[0].numpy())
        scores.append(lg.float().sigmoid()[0].numpy())
        idx.append(i[0].numpy().astype(np.int32))
        wts.append(w[0].float().numpy())
    np.savez_compressed(OUT, logits=np.stack(logits), scores=np.stack(scores), idx=np.stack(idx),
                        wts=np.stack(wts), sha256=np.array(digest(W, xs, bias)),
                        torch=np.array(torch.__version__))
    print("wrote", OUT, os.path.getsize(OUT), "bytes; torch", torch.__version__)


if __name__ == "__main__":
    main()

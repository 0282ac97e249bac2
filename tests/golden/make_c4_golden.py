"""Golden greedy decode of BASELINE config 4 through the REFERENCE's own
layer code (dsv4_layer_forward, compiled from its sources into
oracle/_ref/libdsv4ref.so): the synthetic tiny model of
dsv4_model.tiny_config() with seed 0, a random 32-token prompt (seed 0) and
64 generated tokens. Stores every emitted token, the logits of the first 8
and last 2 emitted positions, and every position's top-1/top-2 margin, in
tests/golden/c4_golden.npz. Needs the reference checkout at build time."""
import os
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(REPO, "oracle"))
sys.path.insert(0, os.path.join(REPO, "deepseek-v4-in-c_b200"))
import oracle as O  # noqa: E402
import dsv4_model as M  # noqa: E402

N_PROMPT, N_GEN, MAX_POS = 32, 64, 256


def prompt(vocab):
    return np.random.default_rng(0).integers(0, vocab, N_PROMPT).astype(np.int32)


def main():
    d = M.tiny_config()
    sm = M.SyntheticModel(d, seed=0)
    toks = prompt(d["vocab"])
    t0 = time.time()
    out, lg = O.model_greedy_ref(sm, toks, N_GEN, MAX_POS)
    print("reference: %d tokens in %.1f s" % (len(out), time.time() - t0))
    srt = np.sort(lg, axis=1)
    margin = srt[:, -1] - srt[:, -2]
    np.savez_compressed(os.path.join(REPO, "tests", "golden", "c4_golden.npz"), prompt=toks, tokens=out,
                        logits_head=lg[:8], logits_tail=lg[-2:], margin=margin)
    print("tokens", out[:16], "... min margin %.3g" % margin.min())


if __name__ == "__main__":
    main()

"""Generate the golden vectors that pin the oracle to the reference.

Runs the REFERENCE's own C (oracle/_ref/libdsv4ref.so, compiled from the
reference sources by `make -C oracle ref`) on seeded inputs and stores inputs
and outputs in tests/golden/golden.npz. tests/test_oracle_golden.py then
requires the restatement (oracle/liboracle.so) to reproduce every output
bit for bit. Needs the reference checkout at build time only; the .npz is
committed so the tests run anywhere.

    python tests/golden/make_golden.py [--full-topk]

--full-topk adds the config-3 sized selection (32768 scores -> top 2048),
which the reference's O(n*k^2) dsv4_topk needs about a minute for.
"""
import argparse
import os
import sys

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(REPO, "oracle"))
sys.path.insert(0, os.path.join(REPO, "deepseek-v4-in-c_b200"))
import oracle as O  # noqa: E402
import dsv4_quant as Q  # noqa: E402

OUT = os.path.join(REPO, "tests", "golden", "golden.npz")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--full-topk", action="store_true")
    a = ap.parse_args()
    ref = O.Checker("reference")
    rng = np.random.default_rng(20261201)
    g = {}

    # FP8 GEMV: varied scales, a ragged shape (partial row and column blocks),
    # and a batch, which per (row, token) must equal the GEMV.
    for name, (rows, cols) in {"fp8a": (256, 384), "fp8r": (200, 300)}.items():
        W, S = Q.random_fp8(rng, rows, cols)
        x = rng.standard_normal(cols * 3).astype(np.float32)
        g[name + "_W"], g[name + "_S"], g[name + "_x"] = W, S, x
        g[name + "_y1"] = ref.gemv_fp8(x[:cols], W, S, rows, cols)
        g[name + "_y3"] = ref.gemv_fp8(x, W, S, rows, cols)
    # config-1 distribution at a reduced size (scales clamp to 2^-10)
    W, S, x = Q.c1_gemv(seed=0, rows=256, cols=1024)
    g["fp8c_W"], g["fp8c_S"], g["fp8c_x"] = W, S, x
    g["fp8c_y"] = ref.gemv_fp8(x, W, S, 256, 1024)

    # FP4 GEMV, packed nibbles, 1x32 scales; and a quantised N(0,0.02) matrix.
    W, S = Q.random_fp4(rng, 128, 512)
    x = rng.standard_normal(512 * 2).astype(np.float32)
    g["fp4a_W"], g["fp4a_S"], g["fp4a_x"] = W, S, x
    g["fp4a_y1"] = ref.gemv_fp4(x[:512], W, S, 128, 512)
    g["fp4a_y2"] = ref.gemv_fp4(x, W, S, 128, 512)
    W, S = Q.quant_fp4(rng.standard_normal((64, 256)).astype(np.float32) * 0.02)
    x = rng.standard_normal(256).astype(np.float32)
    g["fp4q_W"], g["fp4q_S"], g["fp4q_x"] = W, S, x
    g["fp4q_y"] = ref.gemv_fp4(x, W, S, 64, 256)

    # BF16, with a row length that leaves a tail after the 16-lane tree.
    W = Q.bf16_encode(rng.standard_normal((48, 200)).astype(np.float32) * 0.05)
    x = rng.standard_normal(200 * 2).astype(np.float32)
    g["bf16_W"], g["bf16_x"] = W, x
    g["bf16_y1"] = ref.gemv_bf16(x[:200], W, 48, 200)
    g["bf16_y2"] = ref.gemv_bf16(x, W, 48, 200)

    # Elementwise and routing.
    v = rng.standard_normal(2048).astype(np.float32) * 8
    u = rng.standard_normal(2048).astype(np.float32) * 8
    g["sw_g"], g["sw_u"] = v, u
    g["sw_y"] = ref.swiglu(v, u, 10.0)
    w = rng.standard_normal(2048).astype(np.float32)
    g["rms_w"], g["rms_y"] = w, ref.rmsnorm(v, w, 1e-6)
    logits = rng.standard_normal(256).astype(np.float32) * 3
    logits[17] = logits[42]                    # a tie: lower index first
    bias = (rng.standard_normal(256) * 0.1).astype(np.float32)
    g["rt_logits"], g["rt_bias"] = logits, bias
    g["rt_idx"], g["rt_w"] = ref.route(logits, 6, 1.5, bias=bias)
    tid = rng.integers(0, 256, (8, 6)).astype(np.int64)
    g["rt_tid"] = tid
    g["rt_hidx"], g["rt_hw"] = ref.route(logits, 6, 1.5, tid2eid=tid, token_id=5)

    # Indexer scoring on keys widened from e4m3, and the selection.
    q = rng.standard_normal((64, 128)).astype(np.float32)
    kc = Q.e4m3_encode(rng.standard_normal((512, 128)).astype(np.float32))
    hw = rng.standard_normal(64).astype(np.float32)
    g["ix_q"], g["ix_k"], g["ix_w"] = q, kc, hw
    sc = ref.indexer_score(q, Q.e4m3_decode(kc), hw, 64, 128)
    g["ix_score"] = sc
    g["ix_top"] = ref.topk(sc, 200)
    t = np.round(rng.standard_normal(4096) * 4).astype(np.float32)   # many ties
    g["tk_s"], g["tk_idx"] = t, ref.topk(t, 512)
    if a.full_topk:
        t = rng.standard_normal(32768).astype(np.float32)
        g["tkf_s"], g["tkf_idx"] = t, ref.topk(t, 2048)

    # Sparse attention with masked slots and per-head sinks.
    qa = rng.standard_normal((8, 576)).astype(np.float32)
    kv = rng.standard_normal((300, 576)).astype(np.float32)
    idx = rng.permutation(300)[:256].astype(np.int32)
    idx[[3, 77, 200]] = -1
    sink = rng.standard_normal(8).astype(np.float32)
    g["at_q"], g["at_kv"], g["at_idx"], g["at_sink"] = qa, kv, idx, sink
    g["at_o"] = ref.sparse_attn(qa, kv, sink, idx, 1.0 / np.sqrt(np.float32(576)))

    # RoPE tables (dense and YaRN) and an application both ways.
    cs, sn = ref.rope_table(64, 600, 0, 10000.0, 16.0, 32.0, 1.0)
    g["rp_cs_d"], g["rp_sn_d"] = cs, sn
    cs2, sn2 = ref.rope_table(64, 600, 65536, 160000.0, 16.0, 32.0, 1.0)
    g["rp_cs_y"], g["rp_sn_y"] = cs2, sn2
    vv = rng.standard_normal(512).astype(np.float32)
    g["rp_v"] = vv
    g["rp_fwd"] = ref.rope_apply(vv, 64, cs2, sn2, 517, 0)
    g["rp_inv"] = ref.rope_apply(vv, 64, cs2, sn2, 517, 1)

    # mHC pre/post.
    hc, hid = 4, 256
    xh = rng.standard_normal(hc * hid).astype(np.float32)
    fn = (rng.standard_normal(((2 + hc) * hc, hc * hid)) * 0.05).astype(np.float32)
    base = rng.standard_normal((2 + hc) * hc).astype(np.float32)
    scl = np.array([0.5, 0.7, 0.9], np.float32)
    g["hc_x"], g["hc_fn"], g["hc_base"], g["hc_scale"] = xh, fn, base, scl
    y, post, comb = ref.hc_pre(xh, fn, base, scl, hc, hid, 20, 1e-6, 1e-6)
    g["hc_y"], g["hc_post"], g["hc_comb"] = y, post, comb
    blk = rng.standard_normal(hid).astype(np.float32)
    g["hc_blk"] = blk
    g["hc_out"] = ref.hc_post(blk, xh, post, comb, hc, hid)

    # Compressor: ratio 4 (overlap) and ratio 8 over 24 positions.
    for ratio in (4, 8):
        coff = 2 if ratio == 4 else 1
        d = 32
        ape = rng.standard_normal((ratio, coff * d)).astype(np.float32)
        kvs = np.zeros(coff * ratio * coff * d, np.float32)
        scs = np.full(coff * ratio * coff * d, -np.inf, np.float32)
        ins = rng.standard_normal((24, 2, coff * d)).astype(np.float32)
        outs = []
        for pos in range(24):
            r, o = ref.compress_step(ins[pos, 0], ins[pos, 1], ape, kvs, scs, pos, ratio, d)
            if r:
                outs.append(o)
        g["cp%d_ape" % ratio], g["cp%d_in" % ratio] = ape, ins
        g["cp%d_out" % ratio] = np.stack(outs)

    np.savez_compressed(OUT, **g)
    print("wrote", OUT, os.path.getsize(OUT), "bytes,", len(g), "arrays")


if __name__ == "__main__":
    main()

"""The oracle restatement must reproduce the reference BIT FOR BIT.

Golden vectors come from the reference's own C (tests/golden/make_golden.py);
the known-answer cases restate the reference's unit gates
(tests/unit/test_matmul.c, test_indexer.c, test_attn.c, test_quant.c).
CPU only.
"""
import numpy as np
import pytest

import dsv4_quant as Q


def beq(a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape, (a.shape, b.shape)
    assert a.tobytes() == b.tobytes(), "not bit-identical"


@pytest.mark.parametrize("name,rows,cols", [("fp8a", 256, 384), ("fp8r", 200, 300)])
def test_fp8_gemv_golden(port, golden, name, rows, cols):
    W, S, x = golden[name + "_W"], golden[name + "_S"], golden[name + "_x"]
    beq(port.gemv_fp8(x[:cols], W, S, rows, cols), golden[name + "_y1"])
    beq(port.gemv_fp8(x, W, S, rows, cols), golden[name + "_y3"])


def test_fp8_config1_distribution_golden(port, golden):
    beq(port.gemv_fp8(golden["fp8c_x"], golden["fp8c_W"], golden["fp8c_S"], 256, 1024),
        golden["fp8c_y"])
    # every block of the N(0, 0.02) config clamps to 2^-10, E8M0 code 117
    assert np.all(golden["fp8c_S"] == 117)


def test_fp4_gemv_golden(port, golden):
    W, S, x = golden["fp4a_W"], golden["fp4a_S"], golden["fp4a_x"]
    beq(port.gemv_fp4(x[:512], W, S, 128, 512), golden["fp4a_y1"])
    beq(port.gemv_fp4(x, W, S, 128, 512), golden["fp4a_y2"])
    beq(port.gemv_fp4(golden["fp4q_x"], golden["fp4q_W"], golden["fp4q_S"], 64, 256),
        golden["fp4q_y"])


def test_bf16_gemv_golden(port, golden):
    W, x = golden["bf16_W"], golden["bf16_x"]
    beq(port.gemv_bf16(x[:200], W, 48, 200), golden["bf16_y1"])
    beq(port.gemv_bf16(x, W, 48, 200), golden["bf16_y2"])


def test_elementwise_golden(port, golden):
    beq(port.swiglu(golden["sw_g"], golden["sw_u"], 10.0), golden["sw_y"])
    beq(port.rmsnorm(golden["sw_g"], golden["rms_w"], 1e-6), golden["rms_y"])


def test_route_golden(port, golden):
    idx, w = port.route(golden["rt_logits"], 6, 1.5, bias=golden["rt_bias"])
    beq(idx, golden["rt_idx"]); beq(w, golden["rt_w"])
    idx, w = port.route(golden["rt_logits"], 6, 1.5, tid2eid=golden["rt_tid"], token_id=5)
    beq(idx, golden["rt_hidx"]); beq(w, golden["rt_hw"])


def test_route_sigmoid_f32_golden(port):
    """Config 2's router (fp32 GEMV, sigmoid scores, top-6, selection-only
    bias, weights renormalised) against the reference's PyTorch restatement
    (tools/dsv4_ref.py route(score_func="sigmoid"); fixture made by
    tests/golden/make_route_golden.py). The reference C has sqrt-softplus
    scoring only, so this pins the oracle's sigmoid path and f32 router."""
    import os
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    import make_route_golden as MR
    g = np.load(MR.OUT)
    W, xs, bias = MR.inputs()
    assert MR.digest(W, xs, bias) == str(g["sha256"]), "seeded inputs changed"
    for t in range(MR.TRIALS):
        b = bias[t] if t % 2 else None
        # the f32 router GEMV: the oracle's double tree against torch's fp32 linear
        lg = port.gemv_f32(xs[t], W, MR.N_EXPERTS, MR.HIDDEN)
        assert np.max(np.abs(lg - g["logits"][t])) <= 1e-6 * np.max(np.abs(g["logits"][t]))
        # scoring and selection on the reference's own logits
        idx, w, orig = port.route(g["logits"][t], MR.TOPK, 1.0, bias=b, score_func=2, with_scores=True)
        assert list(idx) == list(g["idx"][t])
        ulp = np.abs(orig.view(np.int32).astype(np.int64) - g["scores"][t].view(np.int32).astype(np.int64))
        assert ulp.max() <= 4, ulp.max()                    # expf vs torch's vectorised sigmoid: a few ulp
        assert np.max(np.abs(w - g["wts"][t]) / g["wts"][t]) < 1e-6   # double vs float renormalisation
        # end to end from x: the same selection
        idx2, _ = port.route(lg, MR.TOPK, 1.0, bias=b, score_func=2)
        assert list(idx2) == list(g["idx"][t])


def test_indexer_and_topk_golden(port, golden):
    sc = port.indexer_score(golden["ix_q"], Q.e4m3_decode(golden["ix_k"]),
                            golden["ix_w"], 64, 128)
    beq(sc, golden["ix_score"])
    beq(port.topk(sc, 200), golden["ix_top"])
    beq(port.topk(golden["tk_s"], 512), golden["tk_idx"])
    if "tkf_s" in golden.files:          # the config-3 sized selection
        beq(port.topk(golden["tkf_s"], 2048), golden["tkf_idx"])


def test_sparse_attn_golden(port, golden):
    o = port.sparse_attn(golden["at_q"], golden["at_kv"], golden["at_sink"],
                         golden["at_idx"], 1.0 / np.sqrt(np.float32(576)))
    beq(o, golden["at_o"])


def test_rope_golden(port, golden):
    cs, sn = port.rope_table(64, 600, 0, 10000.0, 16.0, 32.0, 1.0)
    beq(cs, golden["rp_cs_d"]); beq(sn, golden["rp_sn_d"])
    cs, sn = port.rope_table(64, 600, 65536, 160000.0, 16.0, 32.0, 1.0)
    beq(cs, golden["rp_cs_y"]); beq(sn, golden["rp_sn_y"])
    beq(port.rope_apply(golden["rp_v"], 64, cs, sn, 517, 0), golden["rp_fwd"])
    beq(port.rope_apply(golden["rp_v"], 64, cs, sn, 517, 1), golden["rp_inv"])


def test_hc_golden(port, golden):
    y, post, comb = port.hc_pre(golden["hc_x"], golden["hc_fn"], golden["hc_base"],
                                golden["hc_scale"], 4, 256, 20, 1e-6, 1e-6)
    beq(y, golden["hc_y"]); beq(post, golden["hc_post"]); beq(comb, golden["hc_comb"])
    beq(port.hc_post(golden["hc_blk"], golden["hc_x"], post, comb, 4, 256),
        golden["hc_out"])


@pytest.mark.parametrize("ratio", [4, 8])
def test_compressor_golden(port, golden, ratio):
    coff, d = (2 if ratio == 4 else 1), 32
    kvs = np.zeros(coff * ratio * coff * d, np.float32)
    scs = np.full(coff * ratio * coff * d, -np.inf, np.float32)
    ins, ape = golden["cp%d_in" % ratio], golden["cp%d_ape" % ratio]
    outs = []
    for pos in range(ins.shape[0]):
        r, o = port.compress_step(ins[pos, 0], ins[pos, 1], ape, kvs, scs, pos, ratio, d)
        if r:
            outs.append(o)
    beq(np.stack(outs), golden["cp%d_out" % ratio])


# ------------------------------------------------ restated unit known answers

def test_e4m3_all_codes(port):
    """tests/unit/test_quant.c GATE 2 and test_cuda.c GATE 1: all 256 codes."""
    import torch
    codes = np.arange(256, dtype=np.uint8)
    mine = port.e4m3(codes)
    want = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    nan = np.isnan(want)
    assert set(np.nonzero(nan)[0]) == {0x7F, 0xFF}
    assert np.all(np.isnan(mine[nan]))
    assert mine[~nan].tobytes() == want[~nan].tobytes()
    assert Q.e4m3_decode(codes)[~nan].tobytes() == want[~nan].tobytes()


def test_matmul_known_answers(port):
    """tests/unit/test_matmul.c GATES 1-5."""
    W = np.concatenate([np.full(128, 0x38, np.uint8), np.full(128, 0x40, np.uint8)]).reshape(2, 128)
    y = port.gemv_fp8(np.ones(128, np.float32), W, np.array([[128]], np.uint8), 2, 128)
    assert list(y) == [256.0, 512.0]
    y = port.gemv_fp8(np.ones(128, np.float32), np.full((256, 128), 0x38, np.uint8),
                      np.array([[127], [129]], np.uint8), 256, 128)
    assert y[127] == 128.0 and y[128] == 512.0
    y = port.gemv_fp8(np.ones(256, np.float32), np.full((1, 256), 0x38, np.uint8),
                      np.array([[127, 128]], np.uint8), 1, 256)
    assert y[0] == 384.0
    y = port.gemv_fp4(np.ones(64, np.float32), np.full((2, 32), 0x22, np.uint8),
                      np.array([[127, 128], [127, 127]], np.uint8), 2, 64)
    assert list(y) == [96.0, 64.0]
    W = np.stack([np.full(16, 0x22, np.uint8), np.full(16, 0x44, np.uint8)])
    y = port.gemv_fp4(np.ones(32, np.float32), W, np.array([[127], [127]], np.uint8), 2, 32)
    assert list(y) == [32.0, 64.0]
    # low nibble first: 0xA2 = (+1.0 even, -1.0 odd) -> sum of (odd - even)... = -16*2
    y = port.gemv_fp4(np.arange(1, 33, dtype=np.float32), np.full((1, 16), 0xA2, np.uint8),
                      np.array([[128]], np.uint8), 1, 32)
    assert y[0] == -32.0


def test_indexer_known_answers(port):
    """tests/unit/test_indexer.c GATES 1-6."""
    out = port.indexer_score(np.array([[1, 0], [0, 0]], np.float32),
                             np.array([[1, 0], [-1, 0]], np.float32),
                             np.ones(2, np.float32), 2, 2)
    assert out[0] > 0 and out[1] == 0.0
    q = np.zeros((4, 16), np.float32); q[0, 0] = 1
    kv = np.zeros((1, 16), np.float32); kv[0, 0] = 1
    w = np.zeros(4, np.float32); w[0] = 1
    want = np.float32(1 / np.sqrt(np.float32(16))) * np.float32(1 / np.sqrt(np.float32(4)))
    assert abs(port.indexer_score(q, kv, w, 4, 16)[0] - want) < 1e-6
    idx = port.topk(np.array([1, 5, 5, 2, 0, 5], np.float32), 4)
    assert list(idx) == [1, 2, 5, 3]
    assert len(port.topk(np.array([1, 5, 5, 2, 0, 5], np.float32), 10)) == 6
    slots, n = port.window_idxs(5, 4)
    assert n == 4 and list(slots) == [1, 0, 3, 2]
    slots, n = port.window_idxs(2, 4)
    assert n == 3 and list(slots) == [2, 1, 0, -1]


def test_attention_known_answers(port):
    """tests/unit/test_attn.c GATES 1-6."""
    kv = np.repeat(np.arange(1, 5, dtype=np.float32)[:, None], 4, 1)
    o = port.sparse_attn(np.zeros((2, 4), np.float32), kv, np.full(2, -1000, np.float32),
                         np.arange(4, dtype=np.int32), 1.0)
    assert np.allclose(o, 2.5, atol=1e-5)
    o = port.sparse_attn(np.zeros((1, 2), np.float32), np.full((1, 2), 8, np.float32),
                         np.zeros(1, np.float32), np.zeros(1, np.int32), 1.0)
    assert abs(o[0, 0] - 4.0) < 1e-5               # the sink is in the denominator only
    kv2 = np.repeat(np.arange(1, 5, dtype=np.float32)[:, None], 2, 1)
    o = port.sparse_attn(np.zeros((1, 2), np.float32), kv2, np.full(1, -1000, np.float32),
                         np.array([0, -1, 2, -1], np.int32), 1.0)
    assert abs(o[0, 0] - 2.0) < 1e-5               # masked slots contribute nothing
    o = port.sparse_attn(np.zeros((1, 2), np.float32), kv2, np.full(1, 0, np.float32),
                         np.array([-1, -1], np.int32), 1.0)
    assert np.all(o == 0.0)                        # all masked -> zero output


def test_fp4_quantiser_torch_matches_numpy():
    """The torch quantiser the full-size config-2 test runs on the GPU gives
    quant_fp4's codes and scales bit for bit (on CPU torch here), exact
    power-of-two block maxima and ties at the e2m1 midpoints included."""
    import torch
    rng = np.random.default_rng(4)
    w = rng.standard_normal((64, 1024), dtype=np.float32) * np.float32(0.02)
    w[3, :32] = np.float32(0.09375) * np.sign(rng.standard_normal(32)).astype(np.float32)  # absmax/6 = 2^-6
    w[5, 32:64] = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0] * 4, np.float32) * np.float32(2.0 ** -4)
    w[7, 64:96] = 0.0
    W, S = Q.quant_fp4(w)
    Wt, St = Q.quant_fp4_torch(torch.from_numpy(w))
    assert Wt.numpy().tobytes() == W.tobytes()
    assert St.numpy().tobytes() == S.tobytes()

"""GEMV parity on the B200 through the C ABI, against the oracle.

Follows the reference's GPU gate (tests/unit/test_cuda.c): exact device
decoder, vector-scaled relative error <= 1e-5 and argmax identity against the
CPU path, and the batched device path BIT-IDENTICAL to single calls.
"""
import numpy as np
import pytest

import dsv4_b200 as B
import dsv4_quant as Q
from conftest import vrel

pytestmark = pytest.mark.gpu
TOL = 1e-5          # tests/unit/test_cuda.c:186


@pytest.fixture(scope="module")
def dev():
    L = B.init()
    yield L


def test_e4m3_decoder_all_codes(dev, port):
    d = B.dump_e4m3()
    h = port.e4m3(np.arange(256, dtype=np.uint8))
    nan = np.isnan(h)
    assert np.all(np.isnan(d[nan]))
    assert d[~nan].tobytes() == h[~nan].tobytes()


def test_fp8_config1(dev, port):
    """4096x7168, N(0,0.02) in e4m3, 2^-10..2^-4 scales."""
    W, S, x = Q.c1_gemv(seed=0)
    m = B.Matrix(B.WFP8, W, S)
    assert m.upload() == 0 and m.has() == 1
    y = m.mmq(x)
    ref = port.gemv_fp8(x, W, S, 4096, 7168)
    assert vrel(y, ref) < TOL
    assert int(np.argmax(y)) == int(np.argmax(ref))


def test_fp8_varied_scales_batched_bit_identical(dev, port):
    """test_cuda.c GATES 2-4 at its own shape (wo_b 4096x8192), with varied
    scales and per-token-different activations."""
    rng = np.random.default_rng(20260820)
    W, S = Q.random_fp8(rng, 4096, 8192)
    m = B.Matrix(B.WFP8, W, S)
    assert m.upload() == 0
    x = rng.standard_normal(8192).astype(np.float32)
    y = m.mmq(x)
    ref = port.gemv_fp8(x, W, S, 4096, 8192)
    assert vrel(y, ref) < TOL and np.argmax(y) == np.argmax(ref)
    nt = 8
    xn = np.sin(0.7 * (np.arange(8192)[None, :] + 1) + 3.1 * (np.arange(nt)[:, None] + 1)).astype(np.float32)
    yn = m.mmq(xn)
    for t in range(nt):
        assert yn[t].tobytes() == m.mmq(xn[t]).tobytes(), "token %d" % t
    y1 = m.mmq(xn[:1].reshape(-1))
    assert y1.tobytes() == yn[0].tobytes()


@pytest.mark.parametrize("nt", [3, 17, 64])
def test_fp8_batched_against_oracle(dev, port, nt):
    rng = np.random.default_rng(nt)
    W, S = Q.random_fp8(rng, 1024, 4096)
    m = B.Matrix(B.WFP8, W, S)
    assert m.upload() == 0
    xn = rng.standard_normal((nt, 4096)).astype(np.float32)
    yn = m.mmq(xn)
    ref = port.gemv_fp8(xn, W, S, 1024, 4096)
    for t in range(nt):
        assert vrel(yn[t], ref[t]) < TOL
        assert yn[t].tobytes() == m.mmq(xn[t]).tobytes()


def test_fp4_expert_shapes(dev, port):
    rng = np.random.default_rng(4)
    for rows, cols in ((2048, 4096), (4096, 2048)):
        W, S = Q.quant_fp4(rng.standard_normal((rows, cols)).astype(np.float32) * 0.02)
        m = B.Matrix(B.WFP4, W, S)
        assert m.upload() == 0
        x = rng.standard_normal(cols).astype(np.float32)
        assert vrel(m.mmq(x), port.gemv_fp4(x, W, S, rows, cols)) < TOL


def test_bf16_and_f32(dev, port):
    rng = np.random.default_rng(5)
    Wb = Q.bf16_encode(rng.standard_normal((4096, 4096)).astype(np.float32) * 0.02)
    mb = B.Matrix(B.WBF16, Wb)
    assert mb.upload() == 0
    x = rng.standard_normal(4096).astype(np.float32)
    yb = mb.mmq(x)
    rb = port.gemv_bf16(x, Wb, 4096, 4096)
    assert vrel(yb, rb) < TOL and np.argmax(yb) == np.argmax(rb)
    Wf = (rng.standard_normal((256, 4096)) * 0.02).astype(np.float32)
    mf = B.Matrix(B.WF32, Wf)
    assert mf.upload() == 0
    assert vrel(mf.mmq(x), port.gemv_f32(x, Wf, 256, 4096)) < TOL


@pytest.mark.parametrize("fmt,rows,cols", [(B.WFP8, 200, 300), (B.WFP8, 3, 128),
                                           (B.WFP4, 5, 96), (B.WBF16, 7, 200)])
def test_ragged_shapes(dev, port, fmt, rows, cols):
    rng = np.random.default_rng(rows * cols)
    x = rng.standard_normal(cols).astype(np.float32)
    if fmt == B.WFP8:
        W, S = Q.random_fp8(rng, rows, cols)
        ref = port.gemv_fp8(x, W, S, rows, cols)
    elif fmt == B.WFP4:
        W, S = Q.random_fp4(rng, rows, cols)
        ref = port.gemv_fp4(x, W, S, rows, cols)
    else:
        W, S = Q.bf16_encode(rng.standard_normal((rows, cols)).astype(np.float32)), None
        ref = port.gemv_bf16(x, W, rows, cols)
    m = B.Matrix(fmt, W, S, cols=cols)
    assert m.upload() == 0
    assert vrel(m.mmq(x), ref) < TOL


def test_grouped_wo_a_slices_run_on_device(dev, port):
    """dsv4_layer.c:321-334 hands dsv4_mmq row slices of wo_a; the reference
    backend keys residency on the host pointer alone (src/cuda/dsv4_cuda.cu:
    232-241, find(m->w) at :389), so it finds only group 0. Every group must be
    resident here."""
    rng = np.random.default_rng(7)
    G, gr, gw = 8, 1024, 4096
    W, S = Q.random_fp8(rng, G * gr, gw)
    full = B.Matrix(B.WFP8, W, S)
    assert full.upload() == 0
    for gi in range(G):
        sl = full.slice_rows(gi * gr, gr)
        assert sl.has() == 1
        x = rng.standard_normal(gw).astype(np.float32)
        ref = port.gemv_fp8(x, W[gi * gr:(gi + 1) * gr], S[gi * gr // 128:(gi + 1) * gr // 128], gr, gw)
        assert vrel(sl.mmq(x), ref) < TOL
    assert full.slice_rows(64, 128).has() == 0          # not a whole row block


def test_device_api_with_torch_tensors(dev, port):
    import torch
    rng = np.random.default_rng(9)
    W, S = Q.random_fp8(rng, 512, 4096)
    x = rng.standard_normal((2, 4096)).astype(np.float32)
    tW, tS = torch.from_numpy(W).cuda(), torch.from_numpy(S).cuda()
    tx = torch.from_numpy(x).cuda()
    ty = torch.empty((2, 512), dtype=torch.float32, device="cuda")
    B.gemv(B.WFP8, ty, tx, tW, tS, 512, 4096, 128, 128, nt=2,
           stream=torch.cuda.current_stream())
    torch.cuda.synchronize()
    ref = port.gemv_fp8(x, W, S, 512, 4096)
    assert vrel(ty.cpu().numpy(), ref) < TOL


def test_misuse_is_refused(dev):
    bad = B.Matrix(B.WFP8, np.zeros((128, 128), np.uint8), None)   # no scales
    assert bad.upload() == -1 and bad.has() == 0


@pytest.mark.parametrize("fmt,rows,cols", [(B.WFP8, 300, 4000), (B.WBF16, 130, 2000),
                                           (B.WF32, 70, 1000), (B.WFP4, 260, 4096),
                                           (B.WFP8, 16, 16384), (B.WBF16, 1000, 4096)])
def test_single_and_batched_bit_identical_all_formats(dev, port, fmt, rows, cols):
    """Batch-1 calls take the grouped streaming kernel, batched calls the
    nt-token kernel; both sum in the same fixed order, so every token must
    match bitwise.
    Shapes include partial chunks and partial 256-byte segments."""
    rng = np.random.default_rng(rows + cols)
    if fmt == B.WFP8:
        W, S = Q.random_fp8(rng, rows, cols)
    elif fmt == B.WFP4:
        W, S = Q.random_fp4(rng, rows, cols)
    elif fmt == B.WBF16:
        W, S = Q.bf16_encode(rng.standard_normal((rows, cols)).astype(np.float32) * 0.05), None
    else:
        W, S = (rng.standard_normal((rows, cols)) * 0.05).astype(np.float32), None
    m = B.Matrix(fmt, W, S, cols=cols)
    assert m.upload() == 0
    xn = rng.standard_normal((3, cols)).astype(np.float32)
    yn = m.mmq(xn)
    for t in range(3):
        y1 = m.mmq(xn[t])
        assert y1.tobytes() == yn[t].tobytes(), "token %d" % t
        if fmt == B.WFP8:
            ref = port.gemv_fp8(xn[t], W, S, rows, cols)
        elif fmt == B.WFP4:
            ref = port.gemv_fp4(xn[t], W, S, rows, cols)
        elif fmt == B.WBF16:
            ref = port.gemv_bf16(xn[t], W, rows, cols)
        else:
            ref = port.gemv_f32(xn[t], W, rows, cols)
        assert vrel(y1, ref) < TOL

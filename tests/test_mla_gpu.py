"""Sparse MLA decode on the B200 against the oracle.

Indexer scores must be BIT-IDENTICAL to the reference arithmetic
(src/core/dsv4_indexer.c:64-85), the top-k selection identical in members and
order (:92-106: descending, ties to the lower index), and attention
(src/core/dsv4_attn.c:60-108) within 1e-5 of the vector scale.
"""
import numpy as np
import pytest

import dsv4_b200 as B
import dsv4_quant as Q
from conftest import vrel

pytestmark = pytest.mark.gpu
TOL = 1e-5


@pytest.fixture(scope="module")
def dev():
    return B.init()


def c3_sequence(rng, n_pos=32768, H=64, D=576, HI=64, DI=128):
    kv = Q.bf16_encode(rng.standard_normal((n_pos, D), dtype=np.float32))
    keys = Q.e4m3_encode(rng.standard_normal((n_pos, DI), dtype=np.float32))
    q = rng.standard_normal((H, D), dtype=np.float32)
    qi = rng.standard_normal((HI, DI), dtype=np.float32)
    w = rng.standard_normal(HI, dtype=np.float32)
    sink = rng.standard_normal(H, dtype=np.float32)
    return kv, keys, q, qi, w, sink


def bf16_to_f32(u16):
    return (np.asarray(u16, np.uint32) << 16).view(np.float32)


def test_indexer_scores_bit_identical(dev, port):
    rng = np.random.default_rng(31)
    keys = Q.e4m3_decode(Q.e4m3_encode(rng.standard_normal((4096, 128), dtype=np.float32)))
    q = rng.standard_normal((64, 128), dtype=np.float32)
    w = rng.standard_normal(64, dtype=np.float32)
    got = B.indexer_score(q, keys, w)
    ref = port.indexer_score(q, keys, w, 64, 128)
    assert got.tobytes() == ref.tobytes()


@pytest.mark.parametrize("n,k", [(32768, 2048), (5000, 512), (300, 300), (100, 512), (1, 1), (4096, 1)])
def test_topk_exact(dev, port, n, k):
    rng = np.random.default_rng(n + k)
    s = rng.standard_normal(n).astype(np.float32)
    assert list(B.topk(s, k)) == list(port.topk(s, k))


def test_topk_ties_and_signs(dev, port):
    rng = np.random.default_rng(5)
    s = np.round(rng.standard_normal(20000) * 3).astype(np.float32)   # massive ties
    s[::7] = -0.0
    s[3::11] = 0.0
    for k in (1, 17, 2048, 4096):
        assert list(B.topk(s, k)) == list(port.topk(s, k))
    same = np.full(3000, 1.5, np.float32)
    assert list(B.topk(same, 100)) == list(range(100))


def test_sparse_attn_edges(dev, port):
    rng = np.random.default_rng(6)
    q = rng.standard_normal((8, 576), dtype=np.float32)
    kv = rng.standard_normal((500, 576), dtype=np.float32)
    sink = rng.standard_normal(8).astype(np.float32)
    idx = rng.permutation(500)[:300].astype(np.int32)
    idx[[0, 64, 299]] = -1
    sc = 1.0 / np.sqrt(np.float32(576))
    assert vrel(B.sparse_attn(q, kv, sink, idx, sc), port.sparse_attn(q, kv, sink, idx, sc)) < TOL
    allm = np.full(70, -1, np.int32)
    assert np.all(B.sparse_attn(q, kv, sink, allm, sc) == 0.0)
    big = np.full(8, 30.0, np.float32)                  # the sink takes nearly all mass
    assert vrel(B.sparse_attn(q, kv, big, idx, sc), port.sparse_attn(q, kv, big, idx, sc)) < TOL


@pytest.mark.parametrize("batch", [1, 8])
def test_config3_pipeline(dev, port, batch):
    """32768 positions of 512+64 bf16 latent KV, 64 query
    heads, indexer 64x128 with e4m3 keys, top-2048, scale 1/sqrt(576)."""
    import torch
    rng = np.random.default_rng(batch)
    seqs = [c3_sequence(rng) for _ in range(batch)]
    N, H, D, HI, DI, K = 32768, 64, 576, 64, 128, 2048
    kv = torch.from_numpy(np.stack([s[0] for s in seqs]).view(np.int16)).cuda()
    keys = torch.from_numpy(np.stack([s[1] for s in seqs])).cuda()
    q = torch.from_numpy(np.stack([s[2] for s in seqs])).cuda()
    qi = torch.from_numpy(np.stack([s[3] for s in seqs])).cuda()
    w = torch.from_numpy(np.stack([s[4] for s in seqs])).cuda()
    sink = torch.from_numpy(seqs[0][5]).cuda()
    scores = torch.empty((batch, N), dtype=torch.float32, device="cuda")
    idx = torch.empty((batch, K), dtype=torch.int32, device="cuda")
    o = torch.empty((batch, H, D), dtype=torch.float32, device="cuda")
    iscale = np.float32(1 / np.sqrt(np.float32(DI))) * np.float32(1 / np.sqrt(np.float32(HI)))
    scale = float(np.float32(1.0) / np.sqrt(np.float32(D)))
    scratch = torch.empty(B.sparse_attn_scratch(H, D, K, batch), dtype=torch.uint8, device="cuda")
    B.indexer_score_dev(scores, qi, keys, B.E4M3, DI, N * DI, w, HI, DI, N, float(iscale), batch)
    B.topk_dev(idx, scores, N, K, batch)
    B.sparse_attn_dev(o, q, kv, B.BF16, N, sink, idx, H, D, K, scale, batch, scratch)
    torch.cuda.synchronize()
    sc_h, idx_h, o_h = scores.cpu().numpy(), idx.cpu().numpy(), o.cpu().numpy()
    for b in range(batch):               # every sequence of the batch against the oracle
        kvf, kf = bf16_to_f32(seqs[b][0]), Q.e4m3_decode(seqs[b][1])
        rs = port.indexer_score(seqs[b][3], kf, seqs[b][4], HI, DI)
        assert sc_h[b].tobytes() == rs.tobytes()
        ri = port.topk(rs, K)
        assert list(idx_h[b]) == list(ri)
        ro = port.sparse_attn(seqs[b][2], kvf, seqs[0][5], ri, scale)   # sinks: per head, shared
        assert vrel(o_h[b], ro) < TOL, (b, vrel(o_h[b], ro))

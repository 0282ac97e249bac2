"""The multi-rank timing logic of bench.py on CPU: world size 2 over gloo,
each rank contributing its own time, every rank getting the slowest one."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, q):
    import sys
    from datetime import timedelta
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        got = bench.max_over_ranks(dist, 10.0 + 5.0 * rank, device="cpu")
        q.put((rank, got))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = dict(q.get(timeout=10) for _ in range(2))
    assert res == {0: 15.0, 1: 15.0}


def test_decode_bytes_model():
    """The algorithmic bytes of a Flash decode token: every trunk and shared
    matrix once, six routed experts per layer, the head; about 11.1 GB."""
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    import dsv4_model as M
    d = M.flash_config()
    b = bench.decode_bytes_per_token(d, 512)
    assert 11.0e9 < b < 11.3e9
    head = d["vocab"] * d["hidden"] * 2
    experts = len(bench.layer_ratios(d)) * d["topk"] * 13369344
    assert b > head + experts


def test_shard_check_flash():
    """The Flash geometry splits over 1, 2, 4 and 8 GPUs (heads, o_groups,
    wo_a / wo_b FP8 blocks, expert inter slices, vocabulary); a head count
    that does not divide does not."""
    import dsv4_b200 as B
    import dsv4_model as M
    d = M.flash_config()
    cfg = M.ConfigOnly(d).cfg
    for g in (1, 2, 4, 8):
        assert B.shard_check(cfg, g), g
    assert not B.shard_check(cfg, 3)
    assert not B.shard_check(cfg, 16)        # o_groups 8 cannot go over 16 ranks
    d2 = dict(d, n_heads=60)
    assert not B.shard_check(M.ConfigOnly(d2).cfg, 8)


def test_shard_plan_tiles_and_sums():
    """Every rank's share of each split dimension (dsv4b_shard_plan, the
    slices the sharded model is built from) tiles the dimension in rank order,
    a rank's heads, q rows and o_lora rows are exactly its o_groups', and the
    ranks' partial outputs add up to the single-GPU result: the wo_b output
    over o_lora column slices, an expert's FFN over inter slices (SwiGLU is
    per inter element), the LM head's argmax over vocabulary slices."""
    import dsv4_b200 as B
    import dsv4_model as M
    d = dict(M.flash_config(), hidden=256, n_heads=16, head_dim=64, o_groups=8, o_lora=128,
             moe_inter=1024, n_shared=1, vocab=512)
    cfg = M.ConfigOnly(d).cfg
    H, hd, og, ol, dm, I, V = 16, 64, 8, 128, 256, 1024, 512
    hpg = H // og
    rng = np.random.default_rng(5)
    o = rng.standard_normal((H, hd))
    wo_a = rng.standard_normal((og * ol, hpg * hd))
    wo_b = rng.standard_normal((dm, og * ol))
    x = rng.standard_normal(dm)
    w1, w3 = rng.standard_normal((I, dm)), rng.standard_normal((I, dm))
    w2 = rng.standard_normal((dm, I))
    head = rng.standard_normal((V, dm))

    def lat(groups):
        return np.concatenate([wo_a[g * ol:(g + 1) * ol] @ o[g * hpg:(g + 1) * hpg].reshape(-1) for g in groups])

    def ffn(a, b, c):
        g = a @ x
        return c @ (g / (1.0 + np.exp(-g)) * (b @ x))

    full_o = wo_b @ lat(range(og))
    full_f = ffn(w1, w3, w2)
    totals = dict(heads=H, q_rows=H * hd, o_groups=og, o_lora=og * ol, inter=I, shared_inter=I, vocab=V)
    for world in (1, 2, 4, 8):
        plans = [B.shard_plan(cfg, world, r) for r in range(world)]
        assert all(p is not None for p in plans), world
        for k, tot in totals.items():
            pos = 0
            for p in plans:
                assert p[k][0] == pos, (world, k)
                pos += p[k][1]
            assert pos == tot, (world, k)
        acc_o, acc_f, best = np.zeros(dm), np.zeros(dm), []
        for p in plans:
            g0, gn = p["o_groups"]
            assert p["heads"] == (g0 * hpg, gn * hpg)
            assert p["q_rows"] == (g0 * hpg * hd, gn * hpg * hd)
            assert p["o_lora"] == (g0 * ol, gn * ol)
            r0, rn = p["o_lora"]
            acc_o += wo_b[:, r0:r0 + rn] @ lat(range(g0, g0 + gn))
            i0, n = p["inter"]
            acc_f += ffn(w1[i0:i0 + n], w3[i0:i0 + n], w2[:, i0:i0 + n])
            v0, vn = p["vocab"]
            lg = head[v0:v0 + vn] @ x
            j = int(np.argmax(lg))
            best.append((lg[j], v0 + j))
        np.testing.assert_allclose(acc_o, full_o, rtol=1e-10, atol=1e-8)
        np.testing.assert_allclose(acc_f, full_f, rtol=1e-10, atol=1e-8)
        assert max(best, key=lambda t: (t[0], -t[1]))[1] == int(np.argmax(head @ x))
    assert B.shard_plan(cfg, 3, 0) is None
    assert B.shard_plan(cfg, 2, 2) is None

"""The multi-rank timing logic of bench.py on CPU: world size 2 over gloo,
each rank contributing its own time, every rank getting the slowest one."""
import os
import socket

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

"""Sharded decode over 2, 4 and 8 GPUs (one process each): experts split along
their inter dimension, q heads / o_groups and wo_b columns by rank, the LM
head by vocabulary, two sums per layer over NVLink peer memory and one argmax
all-gather per token. Every tensor of a rank is the matching slice of the
single-GPU model of the same seed, so the greedy token stream must be the
single-GPU one. Each world size is skipped when the box has fewer GPUs."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, q):
    import sys
    from datetime import timedelta
    os.environ["DSV4_DEVICE"] = str(rank)
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "deepseek-v4-in-c_b200"))
    import torch.distributed as dist
    import dsv4_b200 as B
    import dsv4_model as M
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        B.init()
        cfg = M.ConfigOnly(M.flash_slice(n_layers=3, n_experts=16, ratios=(4, 128)))
        nid = [B.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(nid, src=0)
        prompt = np.random.default_rng(0).integers(0, cfg.d["vocab"], 12).astype(np.int32)
        m = B.Model(cfg, 64, synthetic_seed=11, rank=rank, world=world, nccl_id=nid[0])
        got = [int(t) for t in m.generate(prompt, 10)]
        m.close()
        ref = None
        if rank == 0:
            m1 = B.Model(cfg, 64, synthetic_seed=11)
            ref = [int(t) for t in m1.generate(prompt, 10)]
            m1.close()
        q.put((rank, got, ref))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_decode_matches_single_gpu(world):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        for p in procs:
            p.join(timeout=600)
            assert p.exitcode == 0
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
    res = {}
    for _ in range(world):
        r, got, ref = q.get(timeout=10)
        res[r] = (got, ref)
    for r in range(1, world):
        assert res[r][0] == res[0][0], "rank %d disagrees" % r
    assert res[0][0] == res[0][1], "sharded %s vs single-GPU %s" % (res[0][0], res[0][1])

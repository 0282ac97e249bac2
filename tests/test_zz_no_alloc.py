"""dsv4b_sparse_attn_static (scratch in a fixed device array) against
dsv4b_sparse_attn (caller scratch), both called through the C ABI.

The file name sorts last so the test also runs after every other GPU test in
the same process; it passes alone in a fresh process as well.
"""
import ctypes as C

import numpy as np
import pytest

import dsv4_b200 as B
from conftest import vrel

pytestmark = pytest.mark.gpu
TOL = 1e-5

_VP, _I, _L, _F = C.c_void_p, C.c_int, C.c_long, C.c_float


def _static_fn():
    fn = C.CDLL(B.LIB_PATH).dsv4b_sparse_attn_static
    fn.argtypes = [_VP, _VP, _VP, _I, _L, _VP, _VP, _I, _I, _I, _F, _I, _VP]
    fn.restype = _I
    return fn


def _case(torch, seed, batch, H, D, N, K):
    g = torch.Generator(device="cpu").manual_seed(seed)
    kv = torch.randn((batch, N, D), generator=g).to(torch.bfloat16).cuda()
    q = torch.randn((batch, H, D), generator=g).cuda()
    sink = torch.randn(H, generator=g).cuda()
    idx = torch.stack([torch.randperm(N, generator=g)[:K] for _ in range(batch)]).to(torch.int32)
    idx[:, ::37] = -1                                      # masked slots
    return kv, q, sink, idx.cuda()


@pytest.mark.parametrize("batch,H,D,N,K", [(1, 64, 576, 4096, 640), (2, 64, 512, 2048, 512)])
def test_static_scratch_matches_caller_scratch(batch, H, D, N, K):
    import torch
    B.init()
    fn = _static_fn()
    assert B.sparse_attn_scratch(H, D, K, batch) <= (8 << 20)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(D)))
    for call in range(2):                                  # two calls in a row, fresh inputs each
        kv, q, sink, idx = _case(torch, 100 * call + batch, batch, H, D, N, K)
        o_static = torch.full((batch, H, D), float("nan"), device="cuda")
        o_ref = torch.empty((batch, H, D), device="cuda")
        rc = fn(o_static.data_ptr(), q.data_ptr(), kv.data_ptr(), B.BF16, N, sink.data_ptr(), idx.data_ptr(),
                H, D, K, scale, batch, None)
        assert rc == 0
        scratch = torch.empty(B.sparse_attn_scratch(H, D, K, batch), dtype=torch.uint8, device="cuda")
        B.sparse_attn_dev(o_ref, q, kv, B.BF16, N, sink, idx, H, D, K, scale, batch, scratch)
        torch.cuda.synchronize()
        a, r = o_static.cpu().numpy(), o_ref.cpu().numpy()
        assert np.isfinite(a).all()
        assert vrel(a, r) < TOL


def test_static_scratch_rejects_oversize():
    import torch
    B.init()
    fn = _static_fn()
    H, D, K = 64, 576, 2048
    batch = 8                                              # 64 chunks x 64 heads x 2316 B x 8 > 8 MiB
    assert B.sparse_attn_scratch(H, D, K, batch) > (8 << 20)
    o = torch.empty((batch, H, D), device="cuda")
    rc = fn(o.data_ptr(), o.data_ptr(), o.data_ptr(), B.F32, 1, o.data_ptr(), o.data_ptr(), H, D, K, 1.0, batch,
            None)
    assert rc == -2

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


def _settled_free(torch):
    """The device's free memory once it has stopped changing. The free figure
    is device-wide: a process that ended just before (the reference's gate
    runs as a subprocess) can still be returning its memory, which would read
    as this process's calls changing it. Polled every 0.2 s until two
    readings agree, for at most 10 s."""
    import time
    last = torch.cuda.mem_get_info()[0]
    for _ in range(50):
        time.sleep(0.2)
        now = torch.cuda.mem_get_info()[0]
        if now == last:
            break
        last = now
    return last


@pytest.mark.parametrize("batch,H,D,N,K", [(1, 64, 576, 4096, 640), (2, 64, 512, 2048, 512)])
def test_static_scratch_matches_caller_scratch(batch, H, D, N, K):
    import torch
    B.init()
    fn = _static_fn()
    assert B.sparse_attn_scratch(H, D, K, batch) <= B.SPARSE_ATTN_STATIC_SCRATCH
    scale = float(np.float32(1.0) / np.sqrt(np.float32(D)))
    # every tensor of both calls exists before the first call, so the device's
    # free memory can show that the calls themselves allocate nothing
    cases = [_case(torch, 100 * call + batch, batch, H, D, N, K) for call in range(2)]
    outs = [torch.full((batch, H, D), float("nan"), device="cuda") for _ in range(2)]
    torch.cuda.synchronize()
    free = [_settled_free(torch)]
    for call in range(2):                                  # two calls in a row, fresh inputs each
        kv, q, sink, idx = cases[call]
        rc = fn(outs[call].data_ptr(), q.data_ptr(), kv.data_ptr(), B.BF16, N, sink.data_ptr(), idx.data_ptr(),
                H, D, K, scale, batch, None)
        assert rc == 0
        torch.cuda.synchronize()
        free.append(torch.cuda.mem_get_info()[0])
    # the first call on a device may load the module holding the fixed array
    # (lazy module loading), which is the array itself plus page rounding;
    # after that no call changes the free memory at all
    assert free[0] - free[1] <= B.SPARSE_ATTN_STATIC_SCRATCH + (4 << 20), free
    assert free[2] == free[1], free
    for call in range(2):
        kv, q, sink, idx = cases[call]
        o_ref = torch.empty((batch, H, D), device="cuda")
        scratch = torch.empty(B.sparse_attn_scratch(H, D, K, batch), dtype=torch.uint8, device="cuda")
        B.sparse_attn_dev(o_ref, q, kv, B.BF16, N, sink, idx, H, D, K, scale, batch, scratch)
        torch.cuda.synchronize()
        a, r = outs[call].cpu().numpy(), o_ref.cpu().numpy()
        assert np.isfinite(a).all()
        assert vrel(a, r) < TOL


def test_static_scratch_rejects_oversize():
    import torch
    B.init()
    fn = _static_fn()
    H, D, K = 64, 576, 2048
    batch = 8                                              # 64 chunks x 64 heads x 2316 B x 8 > 8 MiB
    assert B.sparse_attn_scratch(H, D, K, batch) > B.SPARSE_ATTN_STATIC_SCRATCH
    o = torch.empty((batch, H, D), device="cuda")
    rc = fn(o.data_ptr(), o.data_ptr(), o.data_ptr(), B.F32, 1, o.data_ptr(), o.data_ptr(), H, D, K, 1.0, batch,
            None)
    assert rc == -2
    for bad in ((0, D), (H, 0), (H, -4), (H, 1028), (H, 574)):   # heads / width sparse_attn refuses
        assert fn(o.data_ptr(), o.data_ptr(), o.data_ptr(), B.F32, 1, o.data_ptr(), o.data_ptr(), bad[0], bad[1],
                  K, 1.0, 1, None) == -1


def test_static_scratch_on_a_second_device():
    """One process, device 0 then device 1: the array's address and the
    kernels' shared-memory limit are both per device, so the first call on
    device 1 must set them up there (d = 576 needs the raised limit)."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    B.init()
    fn = _static_fn()
    batch, H, D, N, K = 1, 64, 576, 2048, 512
    scale = float(np.float32(1.0) / np.sqrt(np.float32(D)))
    got = []
    for dev in (0, 1):
        with torch.cuda.device(dev):
            st = torch.cuda.Stream()
            kv, q, sink, idx = [t.to("cuda:%d" % dev) for t in _case(torch, 7, batch, H, D, N, K)]
            o = torch.full((batch, H, D), float("nan"), device="cuda:%d" % dev)
            torch.cuda.synchronize()
            rc = fn(o.data_ptr(), q.data_ptr(), kv.data_ptr(), B.BF16, N, sink.data_ptr(), idx.data_ptr(),
                    H, D, K, scale, batch, st.cuda_stream)
            assert rc == 0
            st.synchronize()
            got.append(o.cpu().numpy())
    assert np.isfinite(got[1]).all()
    assert vrel(got[1], got[0]) < TOL

"""The peer exchange's kernel on one GPU with the other ranks emulated
(dsv4b_peer_selftest): the rank-ordered sum when every rank's vector has
arrived, and -- a rank that never stores, a flag nothing sets -- a wait that
gives up after its poll limit, raises the status word the host reads, and
returns, leaving the context usable. No GPU is faulted or hung: the limit is
a few thousand polls."""
import ctypes as C

import numpy as np
import pytest

import dsv4_b200 as B

pytestmark = pytest.mark.gpu


def _selftest():
    f = C.CDLL(B.LIB_PATH).dsv4b_peer_selftest
    f.argtypes = [C.c_int, C.c_int, C.c_uint, C.c_int, C.c_void_p, C.c_void_p]
    f.restype = C.c_int
    return f


@pytest.mark.parametrize("world", [2, 8])
def test_exchange_sums_in_rank_order(world):
    B.init()
    n = 4096
    rng = np.random.default_rng(world)
    x = rng.standard_normal((world, n)).astype(np.float32)
    x[1, :7] = -0.0                      # a -0.0 is sent as +0.0, not read as "empty"
    out = np.empty(n, np.float32)
    assert _selftest()(world, n, 1 << 20, 1, x.ctypes.data, out.ctypes.data) == 0
    want = x[0].copy()
    for r in range(1, world):
        want = (want + np.where(x[r] == 0, np.float32(0), x[r])).astype(np.float32)
    assert out.tobytes() == want.tobytes()


def test_missing_rank_gives_up_and_reports():
    B.init()
    n, world = 1024, 2
    x = np.ones((world, n), np.float32)
    out = np.empty(n, np.float32)
    assert _selftest()(world, n, 4096, 0, x.ctypes.data, out.ctypes.data) == 1
    # the context is still usable: a complete exchange runs right after
    assert _selftest()(world, n, 1 << 20, 1, x.ctypes.data, out.ctypes.data) == 0
    assert np.all(out == 2.0)

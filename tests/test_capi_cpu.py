"""The C-ABI library loads, exports every symbol include/dsv4_b200.h declares,
and refuses work cleanly without a device. CPU only: no compute calls."""
import ctypes as C

import numpy as np

import dsv4_b200 as B


def test_exports_every_declared_symbol():
    L = B.lib()
    names = B.header_functions()
    assert "dsv4_cuda_mmq" in names and "dsv4b_gemv" in names
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_reference_abi_subset_present():
    """Every symbol the reference host calls (include/dsv4/dsv4_cuda.h:65-99,
    plus dsv4_cuda_dump_e4m3 and dsv4_cuda_set_blocking_sync)."""
    ref = ["dsv4_cuda_available", "dsv4_cuda_init", "dsv4_cuda_upload",
           "dsv4_cuda_has", "dsv4_cuda_mmq", "dsv4_cuda_mmq_n",
           "dsv4_cuda_free_vram", "dsv4_cuda_shutdown", "dsv4_cuda_dump_e4m3",
           "dsv4_cuda_set_blocking_sync"]
    L = B.lib()
    for n in ref:
        assert hasattr(L, n), n


def test_qmat_layout_matches_reference():
    # const void *w, *s; int wdt, rows, cols, blk_r, blk_c  -> 16 + 20 + pad
    assert C.sizeof(B.QMat) == 40
    assert B.QMat.wdt.offset == 16 and B.QMat.blk_c.offset == 32


def test_without_device_nothing_is_resident():
    L = B.lib()
    if L.dsv4_cuda_available():
        return                      # a GPU box: covered by the gpu tests
    m = B.Matrix(B.WFP8, np.zeros((128, 128), np.uint8), np.zeros((1, 1), np.uint8))
    assert m.upload() == -1
    assert m.has() == 0
    assert L.dsv4_cuda_free_vram() == 0


def test_model_calls_refuse_a_null_model():
    """The whole-model entry points check their handle before any device
    work: a null model is refused (-1, or a null stream) on any machine."""
    L = B.lib()
    prompt = np.arange(4, dtype=np.int32)
    out = np.zeros(8, np.int32)
    assert L.dsv4b_model_prefill(None, prompt.ctypes.data, 4, 32) == -1
    assert L.dsv4b_model_generate_prefill(None, prompt.ctypes.data, 4, 2, 32, out.ctypes.data) == -1
    assert L.dsv4b_model_prefill_kernels(None) == -1
    assert not L.dsv4b_model_stream(None)
    assert L.dsv4b_model_begin_batch(None, prompt.ctypes.data, 4) == -1
    assert L.dsv4b_model_decode_batch(None, prompt.ctypes.data, 0, out.ctypes.data) == -1
    assert L.dsv4b_model_n_seq(None) == -1

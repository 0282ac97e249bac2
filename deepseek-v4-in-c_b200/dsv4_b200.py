"""ctypes binding of libdsv4_b200.so (include/dsv4_b200.h).

The product's Python face: the same C ABI the reference's C host links
against, reachable from numpy (host buffers, layer 1) and from torch CUDA
tensors (device pointers, layer 2). There is no CPU fallback: loading fails
loudly when the library is missing, and every call that the C ABI rejects
raises.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdsv4_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "dsv4_b200.h")

WF32, WBF16, WFP8, WFP4 = 0, 1, 2, 3


class QMat(C.Structure):
    """The reference's DSV4QMat (include/dsv4/dsv4.h:208-214)."""
    _fields_ = [("w", C.c_void_p), ("s", C.c_void_p), ("wdt", C.c_int),
                ("rows", C.c_int), ("cols", C.c_int),
                ("blk_r", C.c_int), ("blk_c", C.c_int)]


def build():
    """Compile the library in-tree (nvcc cross-compiles without a GPU)."""
    subprocess.run(["make", "-C", HERE, "-j8"], check=True)
    return LIB_PATH


_lib = None


def lib():
    """Load libdsv4_b200.so once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError("libdsv4_b200.so is not built (run `make -C %s`)" % HERE)
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


def _declare(L):
    vp, i, f, sz = C.c_void_p, C.c_int, C.c_float, C.c_size_t
    qp = C.POINTER(QMat)
    sig = {
        "dsv4_cuda_available": ([], i),
        "dsv4_cuda_init": ([], i),
        "dsv4_cuda_set_blocking_sync": ([], i),
        "dsv4_cuda_upload": ([qp], i),
        "dsv4_cuda_has": ([qp], i),
        "dsv4_cuda_mmq": ([vp, vp, qp], None),
        "dsv4_cuda_mmq_n": ([vp, vp, qp, i], None),
        "dsv4_cuda_free_vram": ([], sz),
        "dsv4_cuda_shutdown": ([], None),
        "dsv4_cuda_dump_e4m3": ([vp], i),
        "dsv4_cuda_evict": ([qp], i),
        "dsv4_cuda_resident_ptrs": ([qp, C.POINTER(vp), C.POINTER(vp)], i),
        "dsv4b_gemv": ([i, vp, vp, vp, vp, i, i, i, i, i, vp], i),
        "dsv4_cuda_moe_prepare": ([qp, vp, qp, i, qp, i, f, i, f], vp),
        "dsv4_cuda_moe": ([vp, vp, vp, vp, vp, vp], i),
        "dsv4_cuda_moe_free": ([vp], None),
        "dsv4b_moe_forward": ([vp, vp, vp, vp], i),
        "dsv4_cuda_indexer_score": ([vp, vp, vp, vp, i, i, i], i),
        "dsv4_cuda_topk": ([vp, vp, i, i], i),
        "dsv4_cuda_sparse_attn": ([vp, vp, vp, vp, vp, i, i, i, f], i),
        "dsv4b_indexer_score": ([vp, vp, vp, i, C.c_long, C.c_long, vp, i, i, i, f, i, vp], i),
        "dsv4b_topk": ([vp, vp, i, i, i, vp], i),
        "dsv4b_sparse_attn_scratch": ([i, i, i, i], sz),
        "dsv4b_sparse_attn": ([vp, vp, vp, i, C.c_long, vp, vp, i, i, i, f, i, vp, sz, vp], i),
        "dsv4_cuda_model_create": ([vp, vp, vp, vp, i], vp),
        "dsv4_cuda_model_begin": ([vp, vp, i], i),
        "dsv4_cuda_model_step": ([vp, vp, vp], i),
        "dsv4_cuda_model_generate": ([vp, vp, i, i, vp], i),
        "dsv4_cuda_model_free": ([vp], None),
        "dsv4b_model_step_async": ([vp, vp], i),
        "dsv4_cuda_model_decode": ([vp, i, i, vp], i),
        "dsv4_cuda_model_create_synthetic": ([vp, i, C.c_ulonglong], vp),
        "dsv4_cuda_model_create_synthetic_batch": ([vp, i, C.c_ulonglong, i], vp),
        "dsv4_cuda_model_create_batch": ([vp, vp, vp, vp, i, i], vp),
        "dsv4b_model_n_seq": ([vp], i),
        "dsv4b_model_begin_batch": ([vp, vp, i], i),
        "dsv4b_model_generate_batch": ([vp, vp, i, i, vp], i),
        "dsv4b_model_decode_batch": ([vp, vp, i, vp], i),
        "dsv4b_model_prefill": ([vp, vp, i, i], i),
        "dsv4b_model_generate_prefill": ([vp, vp, i, i, i, vp], i),
        "dsv4b_model_prefill_kernels": ([vp], i),
        "dsv4b_model_stream": ([vp], vp),
        "dsv4_cuda_model_bytes": ([vp], sz),
        "dsv4_cuda_model_step_kernels": ([vp], i),
        "dsv4b_shard_check": ([vp, i], i),
        "dsv4b_shard_plan": ([vp, i, i, vp], i),
        "dsv4b_model_comm_status": ([vp], i),
        "dsv4b_nccl_id_bytes": ([], sz),
        "dsv4b_nccl_unique_id": ([vp], i),
        "dsv4_cuda_model_create_synthetic_sharded": ([vp, i, C.c_ulonglong, i, i, vp], vp),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes, fn.restype = args, res


def header_functions():
    """Names of every function include/dsv4_b200.h declares."""
    import re
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(dsv4b?_\w+)\s*\(", txt)))


def check(rc, what):
    if rc != 0:
        raise RuntimeError("%s failed (rc=%d)" % (what, rc))


def ptr(a):
    """Address of a numpy array or torch tensor."""
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return a.data_ptr()


def stream_ptr(s=None):
    return None if s is None else s.cuda_stream


# ----------------------------------------------------------- host-side API

class Matrix:
    """A host matrix in one of the checkpoint formats, kept alive while it is
    resident (the backend keys residency on the host pointer, as the
    reference's does)."""

    def __init__(self, wdt, W, S=None, rows=None, cols=None, blk=None):
        self.W = np.ascontiguousarray(W)
        self.S = None if S is None else np.ascontiguousarray(S, dtype=np.uint8)
        if rows is None:
            rows = self.W.shape[0]
        if cols is None:
            cols = {WF32: self.W.shape[1], WBF16: self.W.shape[1],
                    WFP8: self.W.shape[1], WFP4: self.W.shape[1] * 2}[wdt]
        if blk is None:
            blk = {WFP8: (128, 128), WFP4: (1, 32)}.get(wdt, (0, 0))
        self.q = QMat(self.W.ctypes.data, None if self.S is None else self.S.ctypes.data,
                      wdt, rows, cols, blk[0], blk[1])

    def slice_rows(self, r0, nrows):
        """A DSV4QMat of rows [r0, r0+nrows), sharing this matrix's bytes --
        the way the reference layer slices wo_a per group."""
        m = Matrix.__new__(Matrix)
        m.W, m.S = self.W, self.S
        q = self.q
        rb = {WF32: 4 * q.cols, WBF16: 2 * q.cols, WFP8: q.cols, WFP4: q.cols // 2}[q.wdt]
        s = None
        if self.S is not None:
            sc = -(-q.cols // q.blk_c)
            s = self.S.ctypes.data + (r0 // q.blk_r) * sc
        m.q = QMat(self.W.ctypes.data + r0 * rb, s, q.wdt, nrows, q.cols, q.blk_r, q.blk_c)
        return m

    def upload(self):
        rc = lib().dsv4_cuda_upload(C.byref(self.q))
        self._owned = (rc == 0)
        return rc

    def evict(self):
        if getattr(self, "_owned", False):
            self._owned = False
            return lib().dsv4_cuda_evict(C.byref(self.q))
        return -1

    def __del__(self):
        # Residency is keyed on the host address (as in the reference); once
        # this buffer is freed the address may be reused by another matrix.
        try:
            self.evict()
        except Exception:
            pass

    def has(self):
        return lib().dsv4_cuda_has(C.byref(self.q))

    def mmq(self, x):
        x = np.ascontiguousarray(x, np.float32)
        nt = x.size // self.q.cols
        y = np.empty(nt * self.q.rows, np.float32)
        if nt == 1:
            lib().dsv4_cuda_mmq(y.ctypes.data, x.ctypes.data, C.byref(self.q))
        else:
            lib().dsv4_cuda_mmq_n(y.ctypes.data, x.ctypes.data, C.byref(self.q), nt)
        return y.reshape(nt, self.q.rows) if nt > 1 else y

    def device_ptrs(self):
        dw, ds = C.c_void_p(), C.c_void_p()
        check(lib().dsv4_cuda_resident_ptrs(C.byref(self.q), C.byref(dw), C.byref(ds)),
              "dsv4_cuda_resident_ptrs")
        return dw.value, ds.value


def init():
    L = lib()
    if not L.dsv4_cuda_available():
        raise RuntimeError("no CUDA device: the B200 backend has no CPU fallback")
    check(L.dsv4_cuda_init(), "dsv4_cuda_init")
    return L


def dump_e4m3():
    out = np.empty(256, np.float32)
    check(lib().dsv4_cuda_dump_e4m3(out.ctypes.data), "dsv4_cuda_dump_e4m3")
    return out


# ---------------------------------------------------------- device-side API

def gemv(wdt, y, x, W, S, rows, cols, blk_r=0, blk_c=0, nt=1, stream=None):
    check(lib().dsv4b_gemv(wdt, ptr(y), ptr(x), W if isinstance(W, int) else ptr(W),
                           None if S is None else (S if isinstance(S, int) else ptr(S)),
                           rows, cols, blk_r, blk_c, nt, stream_ptr(stream)), "dsv4b_gemv")


class MoE:
    """One layer's MoE bound to resident matrices (dsv4_cuda_moe_prepare)."""

    def __init__(self, gate, experts, shared=None, bias=None, topk=6, route_scale=1.0,
                 score_func=2, swiglu_limit=10.0):
        self.gate, self.experts, self.shared = gate, experts, shared
        n = len(experts)
        self._qs = (QMat * (3 * n))(*[m.q for trio in experts for m in trio])
        self._sh = None if shared is None else (QMat * 3)(*[m.q for m in shared])
        self.bias = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self.topk, self.hidden = topk, gate.q.cols
        self.h = lib().dsv4_cuda_moe_prepare(C.byref(gate.q),
                                             None if self.bias is None else self.bias.ctypes.data,
                                             self._qs, n, self._sh, topk, route_scale, score_func,
                                             swiglu_limit)
        if not self.h:
            raise RuntimeError("dsv4_cuda_moe_prepare failed (matrix not resident or bad shapes)")

    def __call__(self, x, fixed=None):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(self.hidden, np.float32)
        idx = np.empty(self.topk, np.int32)
        w = np.empty(self.topk, np.float32)
        fx = None if fixed is None else np.ascontiguousarray(fixed, np.int32)
        check(lib().dsv4_cuda_moe(self.h, out.ctypes.data, x.ctypes.data,
                                  None if fx is None else fx.ctypes.data, idx.ctypes.data,
                                  w.ctypes.data), "dsv4_cuda_moe")
        return out, idx, w

    def forward_dev(self, out, x, stream=None):
        check(lib().dsv4b_moe_forward(self.h, ptr(out), ptr(x), stream_ptr(stream)), "dsv4b_moe_forward")

    def close(self):
        if self.h:
            lib().dsv4_cuda_moe_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------- sparse MLA

F32, BF16, E4M3 = 0, 1, 2
# DSV4B_SPARSE_ATTN_STATIC_SCRATCH: the fixed device array of dsv4b_sparse_attn_static
SPARSE_ATTN_STATIC_SCRATCH = 8 << 20


def _f(a):
    return np.ascontiguousarray(a, np.float32)


def indexer_score(q, kv, weights):
    """dsv4_cuda_indexer_score: reference signature, host buffers."""
    q, kv, w = _f(q), _f(kv), _f(weights)
    n_heads, head_dim = q.shape
    out = np.empty(kv.shape[0], np.float32)
    check(lib().dsv4_cuda_indexer_score(out.ctypes.data, q.ctypes.data, kv.ctypes.data, w.ctypes.data,
                                        n_heads, head_dim, kv.shape[0]), "dsv4_cuda_indexer_score")
    return out


def topk(scores, k):
    scores = _f(scores)
    idx = np.empty(max(1, min(k, scores.size)), np.int32)
    n = lib().dsv4_cuda_topk(idx.ctypes.data, scores.ctypes.data, scores.size, k)
    if n < 0:
        raise RuntimeError("dsv4_cuda_topk failed")
    return idx[:n]


def sparse_attn(q, kv, sink, idxs, scale):
    q, kv, sink = _f(q), _f(kv), _f(sink)
    idxs = np.ascontiguousarray(idxs, np.int32)
    h, d = q.shape
    o = np.empty((h, d), np.float32)
    check(lib().dsv4_cuda_sparse_attn(o.ctypes.data, q.ctypes.data, kv.ctypes.data, sink.ctypes.data,
                                      idxs.ctypes.data, h, d, idxs.size, scale), "dsv4_cuda_sparse_attn")
    return o


def indexer_score_dev(out, q, keys, key_dt, key_stride, seq_key_stride, w, n_heads, head_dim, n_pos,
                      scale, batch, stream=None):
    check(lib().dsv4b_indexer_score(ptr(out), ptr(q), ptr(keys), key_dt, key_stride, seq_key_stride,
                                    ptr(w), n_heads, head_dim, n_pos, scale, batch, stream_ptr(stream)),
          "dsv4b_indexer_score")


def topk_dev(idx, scores, n, k, batch, stream=None):
    check(lib().dsv4b_topk(ptr(idx), ptr(scores), n, k, batch, stream_ptr(stream)), "dsv4b_topk")


def sparse_attn_scratch(n_heads, d, topk_n, batch):
    return lib().dsv4b_sparse_attn_scratch(n_heads, d, topk_n, batch)


def sparse_attn_dev(o, q, kv, kv_dt, seq_kv_rows, sink, idxs, n_heads, d, topk_n, scale, batch,
                    scratch, stream=None):
    nbytes = scratch.numel() * scratch.element_size()
    check(lib().dsv4b_sparse_attn(ptr(o), ptr(q), ptr(kv), kv_dt, seq_kv_rows, ptr(sink), ptr(idxs),
                                  n_heads, d, topk_n, scale, batch, ptr(scratch), nbytes,
                                  stream_ptr(stream)), "dsv4b_sparse_attn")


# ------------------------------------------------------------- whole model

def nccl_unique_id():
    """A new communicator id (bytes) for a sharded model; rank 0 makes it and
    every rank passes the same bytes to Model(..., nccl_id=...)."""
    buf = C.create_string_buffer(lib().dsv4b_nccl_id_bytes())
    check(lib().dsv4b_nccl_unique_id(buf), "dsv4b_nccl_unique_id")
    return buf.raw


def shard_check(cfg, world):
    """True when a model of ctypes config cfg splits over world GPUs."""
    return lib().dsv4b_shard_check(C.addressof(cfg), int(world)) == 0


# the split dimensions of dsv4b_shard_plan, in its order
SHARD_DIMS = ("heads", "q_rows", "o_groups", "o_lora", "inter", "shared_inter", "vocab")


def shard_plan(cfg, world, rank):
    """{dimension: (first, count)} of rank's share of each split dimension
    (dsv4b_shard_plan), or None when cfg does not split over world GPUs."""
    out = (C.c_int * (2 * len(SHARD_DIMS)))()
    if lib().dsv4b_shard_plan(C.addressof(cfg), int(world), int(rank), out) != len(SHARD_DIMS):
        return None
    return {k: (out[2 * j], out[2 * j + 1]) for j, k in enumerate(SHARD_DIMS)}


class Model:
    """A whole model resident on the device (dsv4_cuda_model_create) from a
    dsv4_model.SyntheticModel or any holder of cfg/mw/layers/experts structs.
    With world > 1 (synthetic only), this rank's share of a model sharded over
    world GPUs (one process per GPU, all stepping in lockstep). With n_seq > 1
    (one GPU), a batch of n_seq sequences stepped together
    (generate_batch / begin_batch / decode_batch)."""

    def __init__(self, sm, max_pos, synthetic_seed=None, rank=0, world=1, nccl_id=None, n_seq=1):
        """sm: a dsv4_model.SyntheticModel (host weights), or with
        synthetic_seed set, any holder of .cfg/.d for an on-device model."""
        self.sm, self.max_pos, self.n_seq = sm, max_pos, n_seq
        self.vocab = sm.d["vocab"]
        if n_seq != 1 and world != 1:
            raise ValueError("a batched model runs on one GPU")
        if synthetic_seed is None:
            if world != 1:
                raise ValueError("sharded models are synthetic (synthetic_seed)")
            self.h = lib().dsv4_cuda_model_create_batch(C.addressof(sm.cfg), C.addressof(sm.mw),
                                                        C.addressof(sm.layers), C.addressof(sm.experts), max_pos,
                                                        int(n_seq))
        elif world == 1:
            self.h = lib().dsv4_cuda_model_create_synthetic_batch(C.addressof(sm.cfg), max_pos, synthetic_seed,
                                                                  int(n_seq))
        else:
            idb = C.create_string_buffer(bytes(nccl_id), len(nccl_id))
            self.h = lib().dsv4_cuda_model_create_synthetic_sharded(C.addressof(sm.cfg), max_pos, synthetic_seed,
                                                                    int(rank), int(world), idb)
        if not self.h:
            raise RuntimeError("model creation failed")

    def decode(self, token, pos):
        nxt = np.zeros(1, np.int32)
        check(lib().dsv4_cuda_model_decode(self.h, int(token), int(pos), nxt.ctypes.data),
              "dsv4_cuda_model_decode")
        return int(nxt[0])

    def device_bytes(self):
        return lib().dsv4_cuda_model_bytes(self.h)

    def begin(self, prompt):
        p = np.ascontiguousarray(prompt, np.int32)
        check(lib().dsv4_cuda_model_begin(self.h, p.ctypes.data, p.size), "dsv4_cuda_model_begin")

    def step(self, want_logits=False):
        tok = np.zeros(1, np.int32)
        lg = np.empty(self.vocab, np.float32) if want_logits else None
        check(lib().dsv4_cuda_model_step(self.h, tok.ctypes.data, None if lg is None else lg.ctypes.data),
              "dsv4_cuda_model_step")
        return int(tok[0]), lg

    def generate(self, prompt, n_gen):
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.empty(n_gen + 1, np.int32)
        n = lib().dsv4_cuda_model_generate(self.h, p.ctypes.data, p.size, n_gen, out.ctypes.data)
        if n < 0:
            raise RuntimeError("dsv4_cuda_model_generate failed")
        return out[:n]

    def prefill(self, prompt, chunk=32):
        """The prompt in passes of chunk tokens; returns the first generated
        token. Steps continue from position len(prompt)."""
        p = np.ascontiguousarray(prompt, np.int32)
        tok = lib().dsv4b_model_prefill(self.h, p.ctypes.data, p.size, int(chunk))
        if tok < 0:
            raise RuntimeError("dsv4b_model_prefill failed")
        return tok

    def generate_prefill(self, prompt, n_gen, chunk=32):
        """generate() with the prompt prefilled in passes of chunk tokens."""
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.empty(n_gen + 1, np.int32)
        n = lib().dsv4b_model_generate_prefill(self.h, p.ctypes.data, p.size, n_gen, int(chunk), out.ctypes.data)
        if n < 0:
            raise RuntimeError("dsv4b_model_generate_prefill failed")
        return out[:n]

    def begin_batch(self, prompts):
        """prompts: [n_seq][n_prompt] int32, one row per sequence."""
        p = np.ascontiguousarray(prompts, np.int32)
        if p.ndim != 2 or p.shape[0] != self.n_seq:
            raise ValueError("prompts must be [n_seq][n_prompt]")
        check(lib().dsv4b_model_begin_batch(self.h, p.ctypes.data, p.shape[1]), "dsv4b_model_begin_batch")

    def generate_batch(self, prompts, n_gen):
        """Greedy tokens [n_seq][n_gen + 1] of every sequence, from its last
        prompt position on."""
        p = np.ascontiguousarray(prompts, np.int32)
        if p.ndim != 2 or p.shape[0] != self.n_seq:
            raise ValueError("prompts must be [n_seq][n_prompt]")
        out = np.empty((self.n_seq, n_gen + 1), np.int32)
        n = lib().dsv4b_model_generate_batch(self.h, p.ctypes.data, p.shape[1], n_gen, out.ctypes.data)
        if n < 0:
            raise RuntimeError("dsv4b_model_generate_batch failed")
        return out[:, :n]

    def decode_batch(self, tokens, pos):
        """Every sequence's token at pos in (host), the next tokens out."""
        t = np.ascontiguousarray(tokens, np.int32)
        nxt = np.zeros(self.n_seq, np.int32)
        check(lib().dsv4b_model_decode_batch(self.h, t.ctypes.data, int(pos), nxt.ctypes.data),
              "dsv4b_model_decode_batch")
        return nxt

    def step_async(self, stream=None):
        check(lib().dsv4b_model_step_async(self.h, stream_ptr(stream)), "dsv4b_model_step_async")

    def close(self):
        if self.h:
            lib().dsv4_cuda_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

"""ctypes bindings for the CPU checkers (TEST INFRASTRUCTURE ONLY).

Two libraries share one set of wrappers:

* ``liboracle.so``  -- the C restatement in oracle/dsv4_oracle.c (prefix
  ``dsv4o_``), always buildable from this repository;
* ``_ref/libdsv4ref.so`` -- the reference's own src/core + src/model C, compiled
  from its sources by ``make -C oracle ref`` (prefix ``dsv4_``). It exists only
  where the reference was present at build time (and travels as a built file).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg import
this module. The product never does.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libdsv4ref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i = C.c_int
_f = C.c_float
_d = C.c_double
_vp = C.c_void_p


def build_oracle():
    """Compile liboracle.so if missing (gcc is present on every box)."""
    if not os.path.exists(ORACLE_SO):
        subprocess.run(["make", "-C", HERE, "liboracle.so"], check=True,
                       stdout=subprocess.DEVNULL)
    return ORACLE_SO


class HcW(C.Structure):
    """Layout of the reference's DSV4HcW (include/dsv4/dsv4.h:266-270)."""
    _fields_ = [("fn", _vp), ("base", _vp), ("scale", _vp)]


class _Lib:
    def __init__(self, path, prefix):
        self.path, self.p = path, prefix
        self.lib = C.CDLL(path)

    def fn(self, name, argtypes, restype=None):
        f = getattr(self.lib, self.p + name)
        f.argtypes, f.restype = argtypes, restype
        return f


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


class Checker:
    """Numpy-level wrappers over one checker library.

    ``kind`` is "port" (the restatement) or "reference" (the reference's own
    C). Functions the reference lacks (f32 GEMV, sigmoid routing) raise
    AttributeError on the reference checker.
    """

    def __init__(self, kind="port"):
        self.kind = kind
        if kind == "port":
            self._l = _Lib(build_oracle(), "dsv4o_")
            self._pre = {"fp8": "gemv_fp8", "fp4": "gemv_fp4", "bf16": "gemv_bf16"}
        else:
            self._l = _Lib(REF_SO, "dsv4_")
            self._pre = {"fp8": "matmul_fp8", "fp4": "matmul_fp4", "bf16": "matmul_bf16"}

    # ---- formats -------------------------------------------------------
    def e4m3(self, b):
        f = self._l.fn("e4m3", [C.c_uint8], _f)
        return np.array([f(int(v)) for v in np.ravel(b)], np.float32)

    # ---- GEMV ----------------------------------------------------------
    def gemv_fp8(self, x, W, S, out, inn, blk_r=128, blk_c=128):
        x = _c(x, np.float32); nt = x.size // inn
        y = np.empty(nt * out, np.float32)
        if nt == 1:
            self._l.fn(self._pre["fp8"], [_f32p, _f32p, _u8p, _u8p, _i, _i, _i, _i])(
                y, x, _c(W, np.uint8), _c(S, np.uint8), inn, out, blk_r, blk_c)
        else:
            self._l.fn(self._pre["fp8"] + "_n", [_f32p, _f32p, _u8p, _u8p, _i, _i, _i, _i, _i])(
                y, x, _c(W, np.uint8), _c(S, np.uint8), inn, out, blk_r, blk_c, nt)
        return y.reshape(nt, out) if nt > 1 else y

    def gemv_fp4(self, x, W, S, out, inn, blk_r=1, blk_c=32):
        x = _c(x, np.float32); nt = x.size // inn
        y = np.empty(nt * out, np.float32)
        if nt == 1:
            self._l.fn(self._pre["fp4"], [_f32p, _f32p, _u8p, _u8p, _i, _i, _i, _i])(
                y, x, _c(W, np.uint8), _c(S, np.uint8), inn, out, blk_r, blk_c)
        else:
            self._l.fn(self._pre["fp4"] + "_n", [_f32p, _f32p, _u8p, _u8p, _i, _i, _i, _i, _i])(
                y, x, _c(W, np.uint8), _c(S, np.uint8), inn, out, blk_r, blk_c, nt)
        return y.reshape(nt, out) if nt > 1 else y

    def gemv_bf16(self, x, W, out, inn):
        x = _c(x, np.float32); nt = x.size // inn
        y = np.empty(nt * out, np.float32)
        if nt == 1:
            self._l.fn(self._pre["bf16"], [_f32p, _f32p, _u16p, _i, _i])(
                y, x, _c(W, np.uint16), inn, out)
        else:
            self._l.fn(self._pre["bf16"] + "_n", [_f32p, _f32p, _u16p, _i, _i, _i])(
                y, x, _c(W, np.uint16), inn, out, nt)
        return y.reshape(nt, out) if nt > 1 else y

    def gemv_f32(self, x, W, out, inn):
        y = np.empty(out, np.float32)
        self._l.fn("gemv_f32", [_f32p, _f32p, _f32p, _i, _i])(
            y, _c(x, np.float32), _c(W, np.float32), inn, out)
        return y

    # ---- elementwise ----------------------------------------------------
    def rmsnorm(self, x, w, eps):
        x = _c(x, np.float32); y = np.empty_like(x)
        self._l.fn("rmsnorm", [_f32p, _f32p, _f32p, _i, _f])(y, x, _c(w, np.float32), x.size, eps)
        return y

    def swiglu(self, g, u, limit):
        g = _c(g, np.float32); y = np.empty_like(g)
        self._l.fn("swiglu", [_f32p, _f32p, _f32p, _i, _f])(y, g, _c(u, np.float32), g.size, limit)
        return y

    def route(self, logits, topk, route_scale, bias=None, tid2eid=None,
              token_id=0, score_func=1, with_scores=False):
        scores = _c(logits, np.float32).copy()
        n = scores.size
        orig = np.empty(n, np.float32)
        idx = np.empty(topk, np.int32); w = np.empty(topk, np.float32)
        bias_p = None if bias is None else _c(bias, np.float32)
        tid_p = None if tid2eid is None else _c(tid2eid, np.int64)
        args = [idx.ctypes.data, w.ctypes.data, scores.ctypes.data, orig.ctypes.data,
                None if bias_p is None else bias_p.ctypes.data,
                None if tid_p is None else tid_p.ctypes.data,
                token_id, n, topk, route_scale]
        at = [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _f]
        if self.kind == "port":
            self._l.fn("route", at + [_i])(*args, score_func)
        else:
            if score_func != 1:
                raise AttributeError("the reference C implements sqrtsoftplus only")
            self._l.fn("route", at)(*args)
        return (idx, w, orig) if with_scores else (idx, w)

    # ---- indexer / attention -------------------------------------------
    def indexer_score(self, q, kv, weights, n_heads, head_dim):
        kv = _c(kv, np.float32); n_pos = kv.size // head_dim
        out = np.empty(n_pos, np.float32)
        self._l.fn("indexer_score", [_f32p, _f32p, _f32p, _f32p, _i, _i, _i])(
            out, _c(q, np.float32), kv, _c(weights, np.float32), n_heads, head_dim, n_pos)
        return out

    def topk(self, scores, k):
        scores = _c(scores, np.float32)
        idx = np.full(max(k, 1), -1, np.int32)
        n = self._l.fn("topk", [_i32p, _f32p, _i, _i], _i)(idx, scores, scores.size, k)
        return idx[:n]

    def sparse_attn(self, q, kv, sink, idxs, scale):
        q = _c(q, np.float32); h, d = q.shape
        idxs = _c(idxs, np.int32)
        o = np.empty((h, d), np.float32)
        scratch = np.empty(h * max(idxs.size, 1), np.float32)
        self._l.fn("sparse_attn", [_f32p, _f32p, _f32p, _f32p, _i32p, _i, _i, _i, _f, _f32p])(
            o, q, _c(kv, np.float32), _c(sink, np.float32), idxs, h, d, idxs.size, scale, scratch)
        return o

    def window_idxs(self, pos, win):
        idx = np.empty(win, np.int32)
        n = self._l.fn("window_idxs", [_i32p, _i, _i], _i)(idx, pos, win)
        return idx, n

    # ---- rope / hc / compressor ------------------------------------------
    def rope_table(self, dim, seqlen, orig, base, factor, bf, bs):
        cs = np.empty(seqlen * (dim // 2), np.float32); sn = np.empty_like(cs)
        self._l.fn("rope_table", [_f32p, _f32p, _i, _i, _i, _d, _d, _d, _d])(
            cs, sn, dim, seqlen, orig, base, factor, bf, bs)
        return cs, sn

    def rope_apply(self, v, rd, cs, sn, pos, inverse):
        v = _c(v, np.float32).copy()
        self._l.fn("rope_apply", [_f32p, _i, _i, _f32p, _f32p, _i, _i, _i])(
            v, v.size, rd, cs, sn, pos, rd // 2, inverse)
        return v

    def hc_pre(self, x, fn, base, scale, hc, hidden, iters, norm_eps, hc_eps):
        y = np.empty(hidden, np.float32); post = np.empty(hc, np.float32)
        comb = np.empty(hc * hc, np.float32); mixes = np.empty((2 + hc) * hc, np.float32)
        x, fn, base, scale = (_c(a, np.float32) for a in (x, fn, base, scale))
        if self.kind == "port":
            self._l.fn("hc_pre", [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                  _i, _i, _i, _f, _f])(
                y, post, comb, mixes, x, fn, base, scale, hc, hidden, iters, norm_eps, hc_eps)
        else:
            w = HcW(fn.ctypes.data, base.ctypes.data, scale.ctypes.data)
            self._l.fn("hc_pre", [_f32p, _f32p, _f32p, _f32p, _f32p, C.POINTER(HcW),
                                  _i, _i, _i, _f, _f])(
                y, post, comb, mixes, x, C.byref(w), hc, hidden, iters, norm_eps, hc_eps)
        return y, post, comb

    def hc_post(self, x, residual, post, comb, hc, hidden):
        y = np.empty(hc * hidden, np.float32)
        self._l.fn("hc_post", [_f32p, _f32p, _f32p, _f32p, _f32p, _i, _i])(
            y, _c(x, np.float32), _c(residual, np.float32), _c(post, np.float32),
            _c(comb, np.float32), hc, hidden)
        return y

    def compress_step(self, kv_in, score_in, ape, kv_state, score_state, pos,
                      ratio, head_dim):
        out = np.zeros(head_dim, np.float32)
        r = self._l.fn("compress_step", [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                         _i, _i, _i], _i)(
            out, _c(kv_in, np.float32), _c(score_in, np.float32), _c(ape, np.float32),
            kv_state, score_state, pos, ratio, head_dim)
        return r, out


class Mat(C.Structure):
    """dsv4o_mat: a DSV4QMat flattened (oracle/dsv4_oracle.h)."""
    _fields_ = [("w", _vp), ("s", _vp), ("wdt", _i), ("rows", _i), ("cols", _i),
                ("blk_r", _i), ("blk_c", _i)]


def mat(wdt, W, S, rows, cols, blk=(0, 0)):
    return Mat(W.ctypes.data, None if S is None else S.ctypes.data, wdt, rows, cols, blk[0], blk[1])


def moe(chk, x, gate, experts, shared, bias, topk, route_scale, score_func, swiglu_limit,
        hidden, inter, inter_shared, fixed=None):
    """dsv4o_moe with dsv4o_mat descriptors (the port only). experts: list of
    (w1, w3, w2) Mat triples; shared: triple or None; fixed: hash-routing row."""
    n = len(experts)
    arr = (Mat * (3 * n))(*[m for t in experts for m in t])
    sh = None if shared is None else (Mat * 3)(*shared)
    out = np.empty(hidden, np.float32)
    idx = np.empty(topk, np.int32); w = np.empty(topk, np.float32)
    x = _c(x, np.float32)
    b = None if bias is None else _c(bias, np.float32)
    tid = None if fixed is None else np.ascontiguousarray(np.asarray(fixed, np.int64).reshape(1, -1))
    f = chk._l.fn("moe", [_f32p, _f32p, C.POINTER(Mat), _vp, _vp, _i, C.POINTER(Mat), C.POINTER(Mat),
                          _i, _i, _f, _i, _i, _i, _i, _f, _i32p, _f32p])
    f(out, x, C.byref(gate), None if b is None else b.ctypes.data,
      None if tid is None else tid.ctypes.data, 0, arr, sh, n, topk, route_scale, score_func,
      hidden, inter, inter_shared, swiglu_limit, idx, w)
    return out, idx, w


def _greedy(step, n_prompt, tokens, n_gen, vocab, keep_logits):
    ids = list(tokens)
    out, rows = [], []
    lg = np.empty(vocab, np.float32)
    for pos in range(n_prompt + n_gen):
        best = step(ids[pos], pos, lg)
        if best < 0:
            raise RuntimeError("model step failed at position %d" % pos)
        if pos + 1 >= n_prompt:
            out.append(best)
            if keep_logits:
                rows.append(lg.copy())
            if pos + 1 < n_prompt + n_gen:
                ids.append(best)
    return np.array(out, np.int32), (np.stack(rows) if keep_logits else None)


def model_greedy_port(sm, tokens, n_gen, max_pos, keep_logits=True):
    """Greedy decode through the oracle's restated model (dsv4_oracle_model.c)."""
    lib = _Lib(build_oracle(), "dsv4o_")
    create = lib.fn("model_create", [_vp, _vp, _vp, _vp, _i], _vp)
    step = lib.fn("model_step", [_vp, _i, _i, _f32p], _i)
    free = lib.fn("model_free", [_vp])
    m = create(C.addressof(sm.cfg), C.addressof(sm.mw), C.addressof(sm.layers), C.addressof(sm.experts),
               max_pos)
    try:
        return _greedy(lambda t, p, lg: step(m, t, p, lg), len(tokens), tokens, n_gen, sm.d["vocab"],
                       keep_logits)
    finally:
        free(m)


def model_greedy_ref(sm, tokens, n_gen, max_pos):
    """Greedy decode through the REFERENCE's dsv4_layer_forward (oracle/_ref)."""
    lib = C.CDLL(REF_SO)
    f = lib.dsv4ref_greedy
    f.argtypes = [_vp, _vp, _vp, _vp, _i, _i32p, _i, _i, _i32p, _f32p]
    f.restype = _i
    toks = np.ascontiguousarray(tokens, np.int32)
    out = np.empty(n_gen + 1, np.int32)
    lg = np.empty((n_gen + 1, sm.d["vocab"]), np.float32)
    n = f(C.addressof(sm.cfg), C.addressof(sm.mw), C.addressof(sm.layers), C.addressof(sm.experts),
          max_pos, toks, toks.size, n_gen, out, lg)
    if n < 0:
        raise RuntimeError("reference driver failed")
    return out[:n], lg[:n]


def model_prefill_ref(sm, tokens, n_gen, max_pos, chunk):
    """The REFERENCE's batched prompt path (oracle/_ref: dsv4_layer_forward_n
    in passes of chunk tokens, dsv4_run.c:391-442), then its per-token loop:
    (the n_gen + 1 greedy tokens from the last prompt position on, the
    seconds of each pass's layer calls, [pass][layer])."""
    lib = C.CDLL(REF_SO)
    f = lib.dsv4ref_prefill_greedy
    f.argtypes = [_vp, _vp, _vp, _vp, _i, _i32p, _i, _i, _i, _i32p,
                  np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")]
    f.restype = _i
    toks = np.ascontiguousarray(tokens, np.int32)
    out = np.empty(n_gen + 1, np.int32)
    tp = np.zeros((-(-toks.size // chunk), sm.d["n_layers"]), np.float64)
    n = f(C.addressof(sm.cfg), C.addressof(sm.mw), C.addressof(sm.layers), C.addressof(sm.experts),
          max_pos, toks, toks.size, n_gen, int(chunk), out, tp)
    if n < 0:
        raise RuntimeError("reference driver failed")
    return out[:n], tp


class BoundCheckpoint:
    """A checkpoint directory bound by the REFERENCE's own reader and binder
    (oracle/_ref: dsv4_st_open, dsv4_bind_model, dsv4_bind_layer, experts by
    their cache's names) into the structs the model constructor takes: .cfg,
    .mw, .layers, .experts, .d (so it stands in for a SyntheticModel)."""

    def __init__(self, directory, sm):
        import dsv4_model as M
        self.d, self.cfg = sm.d, sm.cfg
        nl, ne = sm.d["n_layers"], sm.d["n_experts"]
        self.mw = M.ModelW()
        self.layers = (M.LayerW * nl)()
        self.experts = (M.ExpertW * (nl * ne))()
        self._lib = C.CDLL(REF_SO)
        f = self._lib.dsv4ref_bind_dir
        f.argtypes = [C.c_char_p, _vp, _vp, _vp, _vp]
        f.restype = _vp
        self._lib.dsv4ref_bind_free.argtypes = [_vp]
        self.h = f(os.fsencode(directory), C.addressof(self.cfg), C.addressof(self.mw),
                   C.addressof(self.layers), C.addressof(self.experts))
        if not self.h:
            raise RuntimeError("the reference's binder rejected " + str(directory))

    def close(self):
        if self.h:
            self._lib.dsv4ref_bind_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def model_decode_timed_ref(sm, n_pos, first_token=1, max_pos=None, prompt=None):
    """Per-layer and head wall times (seconds) of the REFERENCE's decode loop
    (dsv4_layer_forward per layer, then hc_head + norm + LM head + argmax)
    over positions 0..n_pos-1 of model sm. With a prompt (int32 tokens), the
    prompt is fed first and n_pos greedy positions follow; the rows then cover
    all len(prompt) + n_pos positions (t_head from len(prompt) - 1 on).
    Returns (t_layer [positions][n_layers], t_head [positions], tokens)."""
    lib = C.CDLL(REF_SO)
    if prompt is not None:
        prompt = np.ascontiguousarray(prompt, np.int32)
        g = lib.dsv4ref_decode_timed_prompt
        g.argtypes = [_vp, _vp, _vp, _vp, _i, _i32p, _i, _i, _i32p,
                      np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS"),
                      np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")]
        g.restype = _i
        npos = len(prompt) + n_pos
        tl = np.zeros((npos, sm.d["n_layers"]), np.float64)
        th = np.zeros(npos, np.float64)
        out = np.empty(n_pos + 1, np.int32)
        n = g(C.addressof(sm.cfg), C.addressof(sm.mw), C.addressof(sm.layers), C.addressof(sm.experts),
              max_pos or npos + 1, prompt, len(prompt), n_pos, out, tl, th)
        if n < 0:
            raise RuntimeError("reference driver failed")
        return tl, th, out[:n]
    f = lib.dsv4ref_decode_timed
    f.argtypes = [_vp, _vp, _vp, _vp, _i, _i, _i, _i32p,
                  np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS"),
                  np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")]
    f.restype = _i
    nl = sm.d["n_layers"]
    tl = np.zeros((n_pos, nl), np.float64)
    th = np.zeros(n_pos, np.float64)
    out = np.empty(n_pos, np.int32)
    n = f(C.addressof(sm.cfg), C.addressof(sm.mw), C.addressof(sm.layers), C.addressof(sm.experts),
          max_pos or n_pos + 1, int(first_token), n_pos, out, tl, th)
    if n < 0:
        raise RuntimeError("reference driver failed")
    return tl, th, out[:n]

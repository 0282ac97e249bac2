"""The reference's model-level structs in ctypes, and synthetic models.

Struct layouts mirror include/dsv4_types.h (itself layout-identical to the
reference's include/dsv4/dsv4.h:94-295, checked by tests/test_layout_cpu.py),
so one set of structs feeds the B200 backend, the oracle and the reference's
own layer code.

`SyntheticModel(cfg, seed)` builds a random-init model of any configuration
in the checkpoint's formats (FP8 128x128 trunk, FP4 1x32 experts, BF16
router / compressor / embeddings / head, f32 norms and mHC), deterministic in
the seed. `tiny_config()` is BASELINE config 4.
"""
import ctypes as C

import numpy as np

import dsv4_quant as Q
from dsv4_b200 import QMat, WF32, WBF16, WFP8, WFP4

_vp, _i, _f = C.c_void_p, C.c_int, C.c_float


class Cfg(C.Structure):
    _fields_ = [(n, _i) for n in ("hidden", "n_layers", "vocab")] + [("rms_eps", _f), ("max_pos", _i)] + \
               [(n, _i) for n in ("n_heads", "n_kv_heads", "head_dim", "q_lora", "o_lora", "o_groups",
                                  "qk_rope", "sliding_window", "index_n_heads", "index_head_dim",
                                  "index_topk", "n_compress")] + \
               [("compress_ratios", C.POINTER(_i)), ("compress_rope_theta", _f),
                ("hc_mult", _i), ("hc_sinkhorn_iters", _i), ("hc_eps", _f),
                ("n_experts", _i), ("topk", _i), ("n_shared", _i), ("moe_inter", _i),
                ("routed_scale", _f), ("norm_topk", _i), ("scoring_func", _i), ("topk_method", _i),
                ("swiglu_limit", _f), ("rope_theta", _f), ("yarn_factor", _f), ("yarn_beta_fast", _f),
                ("yarn_beta_slow", _f), ("yarn_orig_ctx", _i), ("wblock_m", _i), ("wblock_n", _i),
                ("num_hash_layers", _i), ("num_nextn_predict", _i)]


class CompressorW(C.Structure):
    _fields_ = [("ape", _vp), ("norm", _vp), ("wkv", QMat), ("wgate", QMat), ("ratio", _i), ("coff", _i)]


class IndexerW(C.Structure):
    _fields_ = [("wq_b", QMat), ("weights_proj", QMat), ("comp", CompressorW)]


class AttnW(C.Structure):
    _fields_ = [("sink", _vp), ("q_norm", _vp), ("kv_norm", _vp), ("wq_a", QMat), ("wq_b", QMat),
                ("wkv", QMat), ("wo_a", QMat), ("wo_b", QMat), ("comp", CompressorW), ("idx", IndexerW),
                ("has_comp", _i), ("has_idx", _i)]


class ExpertW(C.Structure):
    _fields_ = [("w1", QMat), ("w3", QMat), ("w2", QMat)]


class MoeW(C.Structure):
    _fields_ = [("gate", QMat), ("bias", _vp), ("tid2eid", _vp), ("shared", ExpertW)]


class HcW(C.Structure):
    _fields_ = [("fn", _vp), ("base", _vp), ("scale", _vp)]


class LayerW(C.Structure):
    _fields_ = [("attn_norm", _vp), ("ffn_norm", _vp), ("attn", AttnW), ("moe", MoeW),
                ("hc_attn", HcW), ("hc_ffn", HcW), ("layer", _i), ("compress_ratio", _i),
                ("hash_routed", _i), ("has_comp", _i), ("has_idx", _i)]


class ModelW(C.Structure):
    _fields_ = [("embed", _vp), ("head", _vp), ("norm", _vp), ("hc_head", HcW), ("wdt", _i)]


SCORE_SQRTSOFTPLUS, SCORE_SIGMOID = 1, 2


def tiny_config():
    """4 layers, hidden 1024, 16 heads of 256 latent + 64
    RoPE (head_dim 320), 16 FP4 experts (inter 512) top-2 + 1 shared, vocab
    4096. Choices the config leaves open, recorded here: q_lora 512, o_lora
    256, o_groups 4 (FP8 128x128 blocks stay whole), sliding window 16 (the
    ring wraps within the 96-position run), compress ratios [0, 4, 16, 4] + the
    MTP tail 0 (dense, overlapped-CSA and HCA layers; 16 instead of Flash's 128
    so compressed rows appear within 96 positions), indexer 16 heads x 128
    with index_topk 8 (below the compressed-row count, so selection runs),
    one hash-routed layer, sqrt-softplus scoring as the reference implements."""
    return dict(hidden=1024, n_layers=4, vocab=4096, rms_eps=1e-6, max_pos=256,
                n_heads=16, n_kv_heads=1, head_dim=320, q_lora=512, o_lora=256, o_groups=4,
                qk_rope=64, sliding_window=16, index_n_heads=16, index_head_dim=128, index_topk=8,
                compress_ratios=[0, 4, 16, 4, 0], compress_rope_theta=160000.0,
                hc_mult=4, hc_sinkhorn_iters=20, hc_eps=1e-6,
                n_experts=16, topk=2, n_shared=1, moe_inter=512, routed_scale=1.5, norm_topk=1,
                scoring_func=SCORE_SQRTSOFTPLUS, topk_method=1, swiglu_limit=10.0,
                rope_theta=10000.0, yarn_factor=16.0, yarn_beta_fast=32.0, yarn_beta_slow=1.0,
                yarn_orig_ctx=65536, wblock_m=128, wblock_n=128, num_hash_layers=1,
                num_nextn_predict=1)


def flash_config():
    """The released Flash geometry (reference tests/fixtures/cfg/
    dsv4_flash_config.json), as BASELINE config 5 uses it."""
    return dict(hidden=4096, n_layers=43, vocab=129280, rms_eps=1e-6, max_pos=1048576,
                n_heads=64, n_kv_heads=1, head_dim=512, q_lora=1024, o_lora=1024, o_groups=8,
                qk_rope=64, sliding_window=128, index_n_heads=64, index_head_dim=128, index_topk=512,
                compress_ratios=[0, 0] + [4, 128] * 20 + [4, 0], compress_rope_theta=160000.0,
                hc_mult=4, hc_sinkhorn_iters=20, hc_eps=1e-6,
                n_experts=256, topk=6, n_shared=1, moe_inter=2048, routed_scale=1.5, norm_topk=1,
                scoring_func=SCORE_SQRTSOFTPLUS, topk_method=1, swiglu_limit=10.0,
                rope_theta=10000.0, yarn_factor=16.0, yarn_beta_fast=32.0, yarn_beta_slow=1.0,
                yarn_orig_ctx=65536, wblock_m=128, wblock_n=128, num_hash_layers=3,
                num_nextn_predict=1)


def flash_sample_config():
    """Three layers of the Flash geometry, one of each attention kind
    (compress ratio 0, 4 with the indexer, 128) plus the MTP tail entry, all
    256 experts and the full 129280-token head: the sample the benchmark times
    the reference's CPU decode on and the GPU is checked against."""
    d = flash_config()
    d.update(n_layers=3, compress_ratios=[0, 4, 128, 0], num_hash_layers=1, max_pos=4096)
    return d


def make_cfg(d):
    ratios = (_i * len(d["compress_ratios"]))(*d["compress_ratios"])
    c = Cfg()
    for k, v in d.items():
        if k == "compress_ratios":
            continue
        setattr(c, k, v)
    c.n_compress = d["n_layers"]
    c.compress_ratios = C.cast(ratios, C.POINTER(_i))
    return c, ratios


class SyntheticModel:
    """Random-init weights of a configuration, kept alive with their structs.

    cfg, mw, layers (LayerW * n_layers) and experts (ExpertW * n_layers *
    n_experts, row = layer) are ready for dsv4_cuda_model_create, the oracle's
    dsv4o_model_create and the reference driver."""

    def __init__(self, d, seed=0, sigma=0.02, fast=False):
        """fast=True draws FP8 / FP4 codes uniformly with fixed block scales
        instead of quantising normals: same shapes and formats, for timing
        runs where the values do not matter."""
        self.d = d
        self.fast = fast
        self.rng = np.random.default_rng(seed)
        self.keep = []
        self.cfg, self._ratios = make_cfg(d)
        r = self.rng
        H, hd, hid = d["n_heads"], d["head_dim"], d["hidden"]
        hc = d["hc_mult"]
        mix, hcdim = (2 + hc) * hc, hc * hid
        self.layers = (LayerW * d["n_layers"])()
        self.experts = (ExpertW * (d["n_layers"] * d["n_experts"]))()
        for L in range(d["n_layers"]):
            w = self.layers[L]
            ratio = d["compress_ratios"][L]
            w.layer, w.compress_ratio = L, ratio
            w.hash_routed = 1 if L < d["num_hash_layers"] else 0
            w.has_comp = 1 if ratio != 0 else 0
            w.has_idx = 1 if ratio == 4 else 0
            w.attn_norm = self.f32(1 + 0.1 * r.standard_normal(hid))
            w.ffn_norm = self.f32(1 + 0.1 * r.standard_normal(hid))
            a = w.attn
            a.sink = self.f32(r.standard_normal(H))
            a.q_norm = self.f32(1 + 0.1 * r.standard_normal(d["q_lora"]))
            a.kv_norm = self.f32(1 + 0.1 * r.standard_normal(hd))
            a.wq_a = self.fp8(d["q_lora"], hid, sigma)
            a.wq_b = self.fp8(H * hd, d["q_lora"], sigma)
            a.wkv = self.fp8(hd, hid, sigma)
            a.wo_a = self.fp8(d["o_groups"] * d["o_lora"], H * hd // d["o_groups"], sigma)
            a.wo_b = self.fp8(hid, d["o_groups"] * d["o_lora"], sigma)
            a.has_comp, a.has_idx = w.has_comp, w.has_idx
            if ratio:
                coff = 2 if ratio == 4 else 1
                a.comp = self.compressor(ratio, coff, hd, hid, sigma)
            if ratio == 4:
                a.idx.wq_b = self.fp8(d["index_n_heads"] * d["index_head_dim"], d["q_lora"], sigma)
                a.idx.weights_proj = self.bf16(d["index_n_heads"], hid, sigma)
            m = w.moe
            m.gate = self.bf16(d["n_experts"], hid, sigma)
            if w.hash_routed:
                tid = np.stack([r.permutation(d["n_experts"])[:d["topk"]] for _ in range(d["vocab"])])
                tid = np.ascontiguousarray(tid.astype(np.int64))
                self.keep.append(tid)
                m.tid2eid = tid.ctypes.data
            else:
                m.bias = self.f32(0.05 * r.standard_normal(d["n_experts"]))
            inter_s = d["moe_inter"] * d["n_shared"]
            m.shared.w1 = self.fp8(inter_s, hid, sigma)
            m.shared.w3 = self.fp8(inter_s, hid, sigma)
            m.shared.w2 = self.fp8(hid, inter_s, sigma)
            for e in range(d["n_experts"]):
                ex = self.experts[L * d["n_experts"] + e]
                ex.w1 = self.fp4(d["moe_inter"], hid, sigma)
                ex.w3 = self.fp4(d["moe_inter"], hid, sigma)
                ex.w2 = self.fp4(hid, d["moe_inter"], sigma)
            w.hc_attn = self.hcw(mix, hcdim, 3)
            w.hc_ffn = self.hcw(mix, hcdim, 3)
        self.mw = ModelW()
        self.mw.wdt = WBF16
        self.mw.embed = self.bf16raw(d["vocab"], hid, 1.0)
        self.mw.head = self.bf16raw(d["vocab"], hid, sigma)
        self.mw.norm = self.f32(1 + 0.1 * r.standard_normal(hid))
        self.mw.hc_head = self.hcw(hc, hcdim, 1)

    # ---- helpers -----------------------------------------------------------
    def f32(self, a):
        a = np.ascontiguousarray(a, np.float32)
        self.keep.append(a)
        return a.ctypes.data

    def hcw(self, rows, cols, nscale):
        r = self.rng
        h = HcW()
        h.fn = self.f32(0.02 * r.standard_normal((rows, cols)))
        h.base = self.f32(0.5 * r.standard_normal(rows))
        h.scale = self.f32(0.5 + 0.5 * r.random(nscale))
        return h

    def fp8(self, rows, cols, sigma):
        if self.fast:
            W = self.fast_bytes(rows * cols).reshape(rows, cols) & np.uint8(0xF7)
            S = np.full((-(-rows // 128), -(-cols // 128)), 117, np.uint8)
        else:
            W, S = Q.quant_fp8(self.rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(sigma), 128)
        self.keep += [W, S]
        return QMat(W.ctypes.data, S.ctypes.data, WFP8, rows, cols, 128, 128)

    def fp4(self, rows, cols, sigma):
        if self.fast:
            W = self.fast_bytes(rows * cols // 2).reshape(rows, cols // 2)
            S = np.full((rows, cols // 32), 121, np.uint8)
        else:
            W, S = Q.quant_fp4(self.rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(sigma))
        self.keep += [W, S]
        return QMat(W.ctypes.data, S.ctypes.data, WFP4, rows, cols, 1, 32)

    _POOL = 1 << 26

    def fast_bytes(self, n):
        """n pseudo-random bytes: a window of a 64 MiB random pool at a random
        offset (fast mode; distinct buffers, values irrelevant)."""
        if not hasattr(self, "_pool"):
            self._pool = np.frombuffer(self.rng.bytes(self._POOL), np.uint8)
        out = np.empty(n, np.uint8)
        i = 0
        while i < n:
            off = int(self.rng.integers(0, self._POOL))
            k = min(n - i, self._POOL - off)
            out[i:i + k] = self._pool[off:off + k]
            i += k
        return out

    def bf16raw(self, rows, cols, sigma):
        if self.fast:       # random sign and mantissa, magnitude in [sigma/2, sigma) rounded to a power of 2
            e = int(np.clip(np.floor(np.log2(sigma)) + 127, 1, 254))
            W = (self.fast_bytes(rows * cols * 2).view(np.uint16).reshape(rows, cols)
                 & np.uint16(0x807F)) | np.uint16(e << 7)
        else:
            W = Q.bf16_encode(self.rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(sigma))
        self.keep.append(W)
        return W.ctypes.data

    def bf16(self, rows, cols, sigma):
        return QMat(self.bf16raw(rows, cols, sigma), None, WBF16, rows, cols, 0, 0)

    def compressor(self, ratio, coff, hd, hid, sigma):
        r = self.rng
        cw = CompressorW()
        cw.ratio, cw.coff = ratio, coff
        cw.ape = self.f32(0.1 * r.standard_normal((ratio, coff * hd)))
        cw.norm = self.f32(1 + 0.1 * r.standard_normal(hd))
        cw.wkv = self.bf16(coff * hd, hid, sigma)
        cw.wgate = self.bf16(coff * hd, hid, sigma)
        return cw


class ConfigOnly:
    """Just the config struct of a model, for on-device synthetic models."""

    def __init__(self, d):
        self.d = d
        self.cfg, self._ratios = make_cfg(d)


def flash_slice(n_layers=2, n_experts=16, ratios=(4, 128)):
    """Flash geometry (hidden 4096, 64 heads of 512, indexer 64x128, experts
    2048 wide) cut to a few layers and experts: the shapes of config 5 at a
    size the CPU oracle can still run."""
    d = flash_config()
    d.update(n_layers=n_layers, n_experts=n_experts, compress_ratios=list(ratios) + [0],
             num_hash_layers=1, max_pos=4096)
    return d

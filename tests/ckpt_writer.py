"""A checkpoint directory in the released DeepSeek-V4 safetensors layout,
written from a dsv4_model.SyntheticModel, for the loader test.

Test infrastructure: the names, dtypes and stored shapes are the checkpoint's
(the ones the reference's binder requests, src/model/dsv4_bind.c:66-258, and
its expert cache reads, src/cache/dsv4_cache.c:228-255): FP8 matrices as
F8_E4M3 [rows, cols] with an F8_E8M0 .scale over 128x128 blocks, routed
experts as I8 [rows, cols / 2] (two FP4 codes per byte) with an F8_E8M0
.scale per 32 values, BF16 embedding / head / router / compressor
projections, F32 vectors (the binder widens BF16 or F32 vectors to f32, so
F32 keeps the synthetic values exactly), I64 hash-routing tables."""
import ctypes as C
import json
import os

import numpy as np

_SIZE = {"F32": 4, "BF16": 2, "F8_E4M3": 1, "F8_E8M0": 1, "I8": 1, "I64": 8}


def _qmat(name, q, kind):
    """(name, dtype, shape, get) entries of a quantised pair; get(bundle)
    returns the pointer of the matching field in a (mw, layers, experts)
    bundle."""
    rows, cols = q[0], q[1]
    if kind == "fp8":
        return [(name + ".weight", "F8_E4M3", [rows, cols], "w"),
                (name + ".scale", "F8_E8M0", [-(-rows // 128), -(-cols // 128)], "s")]
    if kind == "fp4":
        return [(name + ".weight", "I8", [rows, cols // 2], "w"),
                (name + ".scale", "F8_E8M0", [rows, cols // 32], "s")]
    return [(name + ".weight", "BF16", [rows, cols], "w")]


def tensor_list(d, layers):
    """Every tensor of the checkpoint of configuration d as (name, dtype,
    shape, path), path locating its pointer in a bundle (mw, layers,
    experts): ("mw", field...), ("L", layer, field...), ("E", layer, expert,
    matrix, "w" | "s")."""
    hid, H, hd = d["hidden"], d["n_heads"], d["head_dim"]
    hc = d["hc_mult"]
    mix, hcd = (2 + hc) * hc, hc * hid
    out = [("embed.weight", "BF16", [d["vocab"], hid], ("mw", "embed")),
           ("norm.weight", "F32", [hid], ("mw", "norm")),
           ("head.weight", "BF16", [d["vocab"], hid], ("mw", "head")),
           ("hc_head_fn", "F32", [hc, hcd], ("mw", "hc_head", "fn")),
           ("hc_head_base", "F32", [hc], ("mw", "hc_head", "base")),
           ("hc_head_scale", "F32", [1], ("mw", "hc_head", "scale"))]

    def q(name, rows, cols, kind, *path):
        for nm, dt, shp, f in _qmat(name, (rows, cols), kind):
            out.append((nm, dt, shp, path + (f,)))

    inter_s = d["moe_inter"] * d["n_shared"]
    for L in range(d["n_layers"]):
        lw = layers[L]
        p = "layers.%d" % L
        out += [(p + ".attn_norm.weight", "F32", [hid], ("L", L, "attn_norm")),
                (p + ".ffn_norm.weight", "F32", [hid], ("L", L, "ffn_norm")),
                (p + ".attn.attn_sink", "F32", [H], ("L", L, "attn", "sink")),
                (p + ".attn.q_norm.weight", "F32", [d["q_lora"]], ("L", L, "attn", "q_norm")),
                (p + ".attn.kv_norm.weight", "F32", [hd], ("L", L, "attn", "kv_norm"))]
        q(p + ".attn.wq_a", d["q_lora"], hid, "fp8", "L", L, "attn", "wq_a")
        q(p + ".attn.wq_b", H * hd, d["q_lora"], "fp8", "L", L, "attn", "wq_b")
        q(p + ".attn.wkv", hd, hid, "fp8", "L", L, "attn", "wkv")
        q(p + ".attn.wo_a", d["o_lora"] * d["o_groups"], H * hd // d["o_groups"], "fp8", "L", L, "attn", "wo_a")
        q(p + ".attn.wo_b", hid, d["o_lora"] * d["o_groups"], "fp8", "L", L, "attn", "wo_b")

        def comp(base, width, *path):
            ratio = lw.compress_ratio
            coff = 2 if ratio == 4 else 1
            out.append((base + ".ape", "F32", [ratio, coff * width], path + ("ape",)))
            out.append((base + ".norm.weight", "F32", [width], path + ("norm",)))
            q(base + ".wkv", coff * width, hid, "bf16", *(path + ("wkv",)))
            q(base + ".wgate", coff * width, hid, "bf16", *(path + ("wgate",)))

        if lw.has_comp:
            comp(p + ".attn.compressor", hd, "L", L, "attn", "comp")
        if lw.has_idx:
            q(p + ".attn.indexer.wq_b", d["index_n_heads"] * d["index_head_dim"], d["q_lora"], "fp8",
              "L", L, "attn", "idx", "wq_b")
            q(p + ".attn.indexer.weights_proj", d["index_n_heads"], hid, "bf16", "L", L, "attn", "idx",
              "weights_proj")
            comp(p + ".attn.indexer.compressor", d["index_head_dim"], "L", L, "attn", "idx", "comp")
        for blk in ("hc_attn", "hc_ffn"):
            out += [("%s.%s_fn" % (p, blk), "F32", [mix, hcd], ("L", L, blk, "fn")),
                    ("%s.%s_base" % (p, blk), "F32", [mix], ("L", L, blk, "base")),
                    ("%s.%s_scale" % (p, blk), "F32", [3], ("L", L, blk, "scale"))]
        q(p + ".ffn.gate", d["n_experts"], hid, "bf16", "L", L, "moe", "gate")
        if lw.hash_routed:
            out.append((p + ".ffn.gate.tid2eid", "I64", [d["vocab"], d["topk"]], ("L", L, "moe", "tid2eid")))
        else:
            out.append((p + ".ffn.gate.bias", "F32", [d["n_experts"]], ("L", L, "moe", "bias")))
        q(p + ".ffn.shared_experts.w1", inter_s, hid, "fp8", "L", L, "moe", "shared", "w1")
        q(p + ".ffn.shared_experts.w3", inter_s, hid, "fp8", "L", L, "moe", "shared", "w3")
        q(p + ".ffn.shared_experts.w2", hid, inter_s, "fp8", "L", L, "moe", "shared", "w2")
        for e in range(d["n_experts"]):
            for w, (rows, cols) in (("w1", (d["moe_inter"], hid)), ("w2", (hid, d["moe_inter"])),
                                    ("w3", (d["moe_inter"], hid))):
                for nm, dt, shp, f in _qmat("%s.ffn.experts.%d.%s" % (p, e, w), (rows, cols), "fp4"):
                    out.append((nm, dt, shp, ("E", L, e, w, f)))
    return out


def nbytes(dtype, shape):
    return int(np.prod(shape)) * _SIZE[dtype]


def resolve(bundle, path, n_experts):
    """The pointer a path names in a bundle (mw, layers, experts)."""
    mw, layers, experts = bundle
    if path[0] == "mw":
        obj, rest = mw, path[1:]
    elif path[0] == "L":
        obj, rest = layers[path[1]], path[2:]
    else:
        obj, rest = experts[path[1] * n_experts + path[2]], path[3:]
    for f in rest:
        obj = getattr(obj, f)
    return obj


def data(bundle, path, n_experts, size):
    """The bytes a path names, or None where the bundle holds no such tensor
    (the synthetic model leaves the indexer's own compressor unset: the
    reference's layer code reads the indexer keys from the main compressor's
    rows, so those tensors are bound but never read)."""
    ptr = resolve(bundle, path, n_experts)
    if not ptr:
        return None
    return np.ctypeslib.as_array((C.c_uint8 * size).from_address(ptr)).copy()


def write_checkpoint(sm, directory):
    """Write sm's weights as one .safetensors file in `directory`; returns
    the tensor list written."""
    d = sm.d
    tl = tensor_list(d, sm.layers)
    bundle = (sm.mw, sm.layers, sm.experts)
    header, chunks, off = {}, [], 0
    for name, dt, shp, path in tl:
        n = nbytes(dt, shp)
        header[name] = {"dtype": dt, "shape": shp, "data_offsets": [off, off + n]}
        v = data(bundle, path, d["n_experts"], n)
        chunks.append(v if v is not None else np.zeros(n, np.uint8))
        off += n
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * (-len(hb) % 8)
    os.makedirs(directory, exist_ok=True)
    with open(os.path.join(directory, "model-00001-of-00001.safetensors"), "wb") as f:
        f.write(np.uint64(len(hb)).tobytes())
        f.write(hb)
        for c in chunks:
            f.write(c.tobytes())
    return tl

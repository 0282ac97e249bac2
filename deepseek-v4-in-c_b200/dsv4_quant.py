"""Host-side packers for the checkpoint's weight formats (numpy).

The formats are the reference's (src/core/dsv4_quant.h:74-164):

* FP8  -- e4m3fn codes, one byte per weight, row-major [rows][cols], with one
  E8M0 scale byte per 128x128 block, grid [ceil(rows/128)][ceil(cols/128)];
* FP4  -- e2m1 codes packed two per byte, the EVEN element in the LOW nibble,
  row-major [rows][cols/2], one E8M0 scale per 1x32 block, grid
  [rows][cols/32];
* BF16 -- the top half of the f32 bit pattern.

Scales are powers of two chosen as 2^ceil(log2(absmax / fmt_max)) (fmt_max 448
for e4m3, 6 for e2m1), optionally clamped to a range, and codes are the
round-to-nearest-even quantisation of w / scale. The synthetic inputs of the
benchmark configurations are built from these.
"""
import numpy as np

E4M3_MAX = 448.0
E2M1_MAX = 6.0


def e8m0_code(scale):
    """Exact E8M0 byte for a power-of-two float scale: 127 + log2(scale)."""
    m, e = np.frexp(np.asarray(scale, np.float64))
    assert np.all(m == 0.5), "E8M0 holds powers of two only"
    return (e - 1 + 127).astype(np.uint8)


def pow2_scale(absmax, fmt_max, lo=None, hi=None):
    """2^ceil(log2(absmax / fmt_max)), with an all-zero block given scale 1."""
    a = np.asarray(absmax, np.float64) / fmt_max
    with np.errstate(divide="ignore"):
        e = np.where(a > 0, np.ceil(np.log2(np.where(a > 0, a, 1.0))), 0.0)
    s = np.exp2(e)
    if lo is not None:
        s = np.maximum(s, lo)
    if hi is not None:
        s = np.minimum(s, hi)
    return s


def e4m3_encode(v):
    """Round-to-nearest-even e4m3fn codes of float values (|v| <= 448)."""
    import torch
    t = torch.from_numpy(np.clip(np.asarray(v, np.float32), -E4M3_MAX, E4M3_MAX))
    return t.to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def e4m3_decode(codes):
    """Exact float of e4m3fn codes (NaN for 0x7F/0xFF)."""
    b = np.asarray(codes, np.uint8).astype(np.int64)
    e, m = (b >> 3) & 15, b & 7
    mag = np.where(e == 0, np.ldexp(m.astype(np.float64), -9),
                   np.ldexp((8 + m).astype(np.float64), (e - 10).astype(np.int32)))
    mag = np.where((e == 15) & (m == 7), np.nan, mag)
    return np.where(b & 0x80, -mag, mag).astype(np.float32)


E2M1_MAG = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float32)


def e2m1_encode(v):
    """Round-to-nearest-even e2m1 4-bit codes (saturating at 6)."""
    v = np.asarray(v, np.float32)
    a = np.abs(v)
    # Midpoints between neighbouring magnitudes; a tie goes to the code whose
    # mantissa bit is 0 (0, 1.0, 2.0, 4.0), i.e. the even code.
    code = np.select(
        [a <= 0.25, a < 0.75, a <= 1.25, a < 1.75, a <= 2.5, a < 3.5, a <= 5.0],
        [0, 1, 2, 3, 4, 5, 6], default=7).astype(np.uint8)
    return code | np.where(v < 0, 8, 0).astype(np.uint8)


def e2m1_decode(codes):
    c = np.asarray(codes, np.uint8)
    mag = E2M1_MAG[c & 7]
    return np.where(c & 8, -mag, mag).astype(np.float32)


def bf16_encode(v):
    import torch
    t = torch.from_numpy(np.asarray(v, np.float32)).to(torch.bfloat16)
    return t.view(torch.int16).numpy().view(np.uint16)


def quant_fp8(w, blk=128, scale_lo=None, scale_hi=None):
    """[rows][cols] float -> (codes [rows][cols] u8, scales [rb][cb] u8)."""
    w = np.asarray(w, np.float32)
    rows, cols = w.shape
    rb, cb = -(-rows // blk), -(-cols // blk)
    pad = np.zeros((rb * blk, cb * blk), np.float32)
    pad[:rows, :cols] = w
    blocks = pad.reshape(rb, blk, cb, blk)
    amax = np.abs(blocks).max(axis=(1, 3))
    s = pow2_scale(amax, E4M3_MAX, scale_lo, scale_hi)
    q = blocks / s[:, None, :, None].astype(np.float32)
    codes = e4m3_encode(q).reshape(rb * blk, cb * blk)[:rows, :cols]
    return np.ascontiguousarray(codes), e8m0_code(s)


def quant_fp4(w, blk=32):
    """[rows][cols] float -> (packed [rows][cols/2] u8, scales [rows][cols/32])."""
    w = np.asarray(w, np.float32)
    rows, cols = w.shape
    assert cols % blk == 0 and cols % 2 == 0
    b = w.reshape(rows, cols // blk, blk)
    s = pow2_scale(np.abs(b).max(axis=2), E2M1_MAX)
    codes = e2m1_encode(b / s[:, :, None].astype(np.float32)).reshape(rows, cols)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    return np.ascontiguousarray(packed), e8m0_code(s)


def quant_fp4_torch(w, blk=32):
    """quant_fp4 on a torch tensor, on whatever device it lives (the config-2
    experts are 6.4 G weights, quantised on the GPU for the tests): the same
    codes and scales bit for bit. The scale exponent comes from frexp, which
    equals ceil(log2(absmax / 6)) for every float32 absmax."""
    import torch
    rows, cols = w.shape
    assert cols % blk == 0 and cols % 2 == 0
    b = w.float().reshape(rows, cols // blk, blk)
    a = b.abs().amax(dim=2).double() / E2M1_MAX
    m, e = torch.frexp(a)
    e = torch.where(a > 0, torch.where(m == 0.5, e - 1, e), torch.zeros_like(e)).to(torch.int32)
    s = torch.ldexp(torch.ones_like(a), e).float()
    q = b / s[:, :, None]
    v = q.abs()
    code = ((v > 0.25).to(torch.uint8) + (v >= 0.75).to(torch.uint8) + (v > 1.25).to(torch.uint8) +
            (v >= 1.75).to(torch.uint8) + (v > 2.5).to(torch.uint8) + (v >= 3.5).to(torch.uint8) +
            (v > 5.0).to(torch.uint8))
    code = (code | torch.where(q < 0, 8, 0).to(torch.uint8)).reshape(rows, cols)
    packed = code[:, 0::2] | (code[:, 1::2] << 4)
    return packed.contiguous(), (e + 127).to(torch.uint8).contiguous()


def dequant_fp8(codes, scales, blk=128):
    v = e4m3_decode(codes).astype(np.float64)
    rows, cols = v.shape
    s = np.exp2(scales.astype(np.float64) - 127)
    return v * np.repeat(np.repeat(s, blk, 0), blk, 1)[:rows, :cols]


def dequant_fp4(packed, scales, blk=32):
    rows = packed.shape[0]
    codes = np.empty((rows, packed.shape[1] * 2), np.uint8)
    codes[:, 0::2] = packed & 15
    codes[:, 1::2] = packed >> 4
    v = e2m1_decode(codes).astype(np.float64)
    return v * np.repeat(np.exp2(scales.astype(np.float64) - 127), blk, 1)


# --------------------------------------------------- benchmark-config inputs

def c1_gemv(seed=0, rows=4096, cols=7168, sigma=0.02):
    """Config 1: W ~ N(0, 0.02) in e4m3 with power-of-two 128x128 block
    scales clamped to [2^-10, 2^-4]; x ~ N(0, 1) f32."""
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(sigma)
    W, S = quant_fp8(w, 128, 2.0 ** -10, 2.0 ** -4)
    x = rng.standard_normal(cols, dtype=np.float32)
    return W, S, x


def random_fp8(rng, rows, cols, scale_lo=120, scale_hi=134):
    """FP8 codes drawn uniformly (NaN codes excluded) with VARIED block scales:
    the correctness-only variant, since constant scales hide scale-indexing
    bugs (reference tests/unit/test_cuda.c:131-138)."""
    W = rng.integers(0, 256, (rows, cols), dtype=np.uint8)
    W[(W & 0x7F) == 0x7F] &= 0xFE
    S = rng.integers(scale_lo, scale_hi + 1, (-(-rows // 128), -(-cols // 128)),
                     dtype=np.uint8)
    return W, S


def random_fp4(rng, rows, cols, scale_lo=118, scale_hi=124):
    """FP4 packed bytes drawn uniformly, with per-32 scales from a range."""
    W = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    S = rng.integers(scale_lo, scale_hi + 1, (rows, cols // 32), dtype=np.uint8)
    return W, S

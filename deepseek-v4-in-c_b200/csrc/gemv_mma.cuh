// gemv_mma.cuh - batch-1 GEMV of FP8 (e4m3, 128x128 E8M0 blocks), FP4 (e2m1,
// 1x32 E8M0 blocks) and BF16 weights on the tensor cores: warp-level mma.sync
// m16n8k16, f32 accumulate.
//
// The weights are the A operand: e4m3 codes widen exactly to f16 (one cvt
// per pair); e2m1 codes are placed in f16 bit fields (e2m1_word) and
// multiplied by their block scale, exact while the scale exponent lies in
// [-23, 1]; bf16 weights are used as they are. x is the B operand, split
// into three pieces that add back to x exactly enough for an f32 dot:
//   f16 paths: xs = x * 2^k (k per unit, so that max|xs| lies in
//              [2^14, 2^15)), hi = f16(xs), lo = f16(xs - hi),
//              lo2 = f16(xs - hi - lo);
//   BF16 path: hi = bf16(x), lo = bf16(x - hi), lo2 = bf16(x - hi - lo).
// The pieces occupy B columns n = 0, 1, 2; every product is exact.
//
// Order (the canonical one for these formats, used by every kernel that
// computes them): a row is cut into units of 128 columns (256 for FP4). For
// each unit b the tensor core accumulates, from zero, the unit's k16-steps
// into C[n]; q_b = (((C[0] + C[1]) + C[2]) * 2^-k) * scale_b in float (FP4:
// the scales are already in A, scale_b = 1); the units are cut into eight
// contiguous runs of ceil(nb / 8), each run summed from zero in double in
// unit order, the eight run sums added in order in double; y = (float)total.
//
// Work: a block of 8 warps streams a tile of rows (a multiple of 16); a unit
// is 16 rows x one 128-column block; the eight contiguous runs of ceil(nb / 8)
// units of the canonical order are shared out among the warps (a warp, or
// with fewer than eight runs a set of warps over alternate row groups, per
// run) and each keeps its run sums itself. Lane
// (g = lane/4, t = lane%4) loads rows g and g+8 at bytes 64 j + 16 t of the
// unit row (chunks j = 0..CPL-1) through a ring of cp.async stages it alone
// reads back; the k index inside a unit is permuted (the dot product does not
// care) so that these 16-byte chunks are exactly the lane's A fragments.
#pragma once

#include "gemv_core.cuh"
#include "internal.h"

namespace dsv4b {

constexpr int kMmaMaxBlocks = 64;                           // blocks per row
constexpr int kMmaStages = 3;                               // ring steps in flight + 1
constexpr int kMmaRing = kMmaStages * 4 * 16 * 256;         // 4 chunks of 16 B per lane per step
constexpr int kMmaSRing = 8 * kMmaStages * 8 * 16;          // FP4 scales: per warp, step and row pair, 16 B
constexpr int kMmaXpPerMma = 12 * 8;                        // x fragment bytes per mma: (t, piece)

template <int FMT> struct MmaFmt;
// E: elements per 16 bytes; CPL: 16-byte chunks per lane and row in a unit;
// STEPS: ring steps per unit (two chunks per row and step); COLS: columns of
// a unit (one flush block); MPU: k16 steps per unit.
template <> struct MmaFmt<DSV4B_WFP8> { static constexpr int E = 16, CPL = 2, STEPS = 1, COLS = 128, MPU = 8; };
template <> struct MmaFmt<DSV4B_WBF16> { static constexpr int E = 8, CPL = 4, STEPS = 2, COLS = 128, MPU = 8; };
template <> struct MmaFmt<DSV4B_WFP4> { static constexpr int E = 32, CPL = 2, STEPS = 1, COLS = 256, MPU = 16; };

__host__ __device__ inline int mma_unit_cols(int fmt) { return fmt == DSV4B_WFP4 ? 256 : 128; }
__host__ __device__ inline int mma_unit_mmas(int fmt) { return fmt == DSV4B_WFP4 ? 16 : 8; }

// Dynamic shared memory of a tile of tr virtual rows over nb units: the
// ring, the FP4 scale ring, the x fragments, the per-unit exponents and the
// eight run sums (double) of every virtual row.
__host__ __device__ inline size_t mma_smem(int fmt, int nb, int tr, int nt = 1)
{
    return (size_t)kMmaRing + kMmaSRing + (size_t)nt * nb * mma_unit_mmas(fmt) * kMmaXpPerMma +
           (((size_t)nt * nb * 4 + 15) & ~(size_t)15) + (size_t)nt * tr * 8 * 8;
}

__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Two e4m3 codes (low byte first) -> f16x2 bits, exact.
__device__ __forceinline__ uint32_t e4m3x2_h2(uint32_t v)
{
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(v & 0xFFFFu), __NV_E4M3);
    return (uint32_t)h.x | ((uint32_t)h.y << 16);
}

// The four f16x2 pairs of a word of eight e2m1 codes (nibble 0 lowest):
// r[q] = (value(q), value(q + 4)) * 2^-14, exactly. An e2m1 code s|e1 e0|m
// placed at f16 bits 15, 11..9 (sign, exponent low bits, mantissa top bit)
// reads as 2^(e-15) (1 + m/2) for e > 0 and as the subnormal m 2^-15 for
// e = 0, i.e. the code's value times 2^-14 in both cases. Only the high byte
// of each f16 is non-zero: (s << 7) | (e1 e0 m << 1). Two masked shifts give
// those bytes for the low and for the high nibbles of the four bytes, and one
// byte permute per pair puts two of them in place.
__device__ __forceinline__ void e2m1_word(uint32_t w, uint32_t (&r)[4])
{
    const uint32_t lo = ((w << 1) & 0x0E0E0E0Eu) | ((w << 4) & 0x80808080u);   // nibbles 0, 2, 4, 6
    const uint32_t hi = ((w >> 3) & 0x0E0E0E0Eu) | (w & 0x80808080u);          // nibbles 1, 3, 5, 7
    r[0] = __byte_perm(lo, 0u, 0x2404);     // nibbles 0, 4
    r[1] = __byte_perm(hi, 0u, 0x2404);     // 1, 5
    r[2] = __byte_perm(lo, 0u, 0x3414);     // 2, 6
    r[3] = __byte_perm(hi, 0u, 0x3414);     // 3, 7
}

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b)
{
    uint32_t o;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o) : "r"(a), "r"(b));
    return o;
}

// E8M0 byte b (scale 2^e, e = b - 127) -> the f16x2 pair (2^(e+14), 2^(e+14)),
// the multiplier that turns an e2m1_word() pair into value * 2^e. Called only for
// e in [-23, 1]: the multiplier is a normal f16 and every code times 2^e is an
// exact f16 (0.5 * 2^-23 = 2^-24 is the smallest subnormal).
__device__ __forceinline__ uint32_t e8m0_h2x(uint32_t b)
{
    const uint32_t h = (b - 98u) << 10;
    return h | (h << 16);
}

// 2^e as a float for e in [-126, 127].
__device__ __forceinline__ float pow2f(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }

// The three pieces of four x values, as f16x2 (x pre-scaled by a power of
// two) or bf16x2 pairs: out[p] = {pair(e0, e1), pair(e2, e3)}.
template <bool BF>
__device__ __forceinline__ void x_pieces(const float4 &x, float sc, uint2 (&out)[3])
{
    const float v[4] = {x.x * sc, x.y * sc, x.z * sc, x.w * sc};   // sc is a power of two: exact
    uint16_t p[3][4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
        if constexpr (!BF) {
            const __half h0 = __float2half_rn(v[e]);
            const float r1 = __fsub_rn(v[e], __half2float(h0));
            const __half h1 = __float2half_rn(r1);
            const __half h2 = __float2half_rn(__fsub_rn(r1, __half2float(h1)));
            p[0][e] = __half_as_ushort(h0);
            p[1][e] = __half_as_ushort(h1);
            p[2][e] = __half_as_ushort(h2);
        } else {
            const __nv_bfloat16 h0 = __float2bfloat16_rn(v[e]);
            const float r1 = __fsub_rn(v[e], __bfloat162float(h0));
            const __nv_bfloat16 h1 = __float2bfloat16_rn(r1);
            const __nv_bfloat16 h2 = __float2bfloat16_rn(__fsub_rn(r1, __bfloat162float(h1)));
            p[0][e] = __bfloat16_as_ushort(h0);
            p[1][e] = __bfloat16_as_ushort(h1);
            p[2][e] = __bfloat16_as_ushort(h2);
        }
    }
#pragma unroll
    for (int q = 0; q < 3; q++)
        out[q] = make_uint2((uint32_t)p[q][0] | ((uint32_t)p[q][1] << 16), (uint32_t)p[q][2] | ((uint32_t)p[q][3] << 16));
}

// NP token pairs per item (it.nt <= 2 NP tokens, x / y it.xts / it.yts
// floats apart): the two tokens of a pair share every mma, token 2p in B
// columns 0-2 and token 2p+1 in columns 3-5. The tensor core forms each
// column from that column's operands alone, so a token's result is the one
// it gets on its own; the weights are streamed and decoded once per item.
// NP = 0: exactly one token (batch-1 launches), the pair logic compiled out.
template <int FMT, int NP>
__device__ __forceinline__ void mma_tile(const GemvItem &it, int tile, unsigned char *smem)
{
    using F = MmaFmt<FMT>;
    constexpr int E = F::E, STEPS = F::STEPS, MPC = E / 4, MPU = F::MPU, UB = F::COLS * 16 / E;   // unit bytes/row
    constexpr bool BF = FMT == DSV4B_WBF16;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int nb = it.cols / F::COLS, rb = it.rowbytes, trh = it.tr >> 1;
    constexpr int NPP = NP > 0 ? NP : 1;                 // accumulator sets
    constexpr int MAXT = NP > 0 ? 2 * NP : 1;           // tokens an item can carry
    int nt = NP > 0 && it.nt > 1 ? it.nt : 1;
    const size_t xtab = (size_t)nb * MPU * 12;            // one token's x fragments (uint2)
    uint4 *ring = reinterpret_cast<uint4 *>(smem);
    uint2 *sring = reinterpret_cast<uint2 *>(smem + kMmaRing);
    uint2 *xp = reinterpret_cast<uint2 *>(smem + kMmaRing + kMmaSRing);                         // [nt][...]

    const uint8_t *W = it.W, *S = it.S, *W2 = it.W2, *S2 = it.S2;
    const float *X = it.x;
    float *Y = it.y;
    // token i's x / y: X + xo[i], Y + yo[i]
    size_t xo[MAXT], yo[MAXT];
#pragma unroll
    for (int i = 0; i < MAXT; i++) {
        xo[i] = (size_t)i * it.xts;
        yo[i] = (size_t)i * it.yts;
    }
    if (it.wtab) {
        pdl_wait();                  // the selection comes from the previous kernel
        int si = it.slot;
        if (it.perm) {
            // a batch's routed group: perm[5 slot] tokens (0 = an unused slot)
            // of one expert, entries (token << 8) | k
            const int *gd = it.perm + (size_t)it.slot * 5;
            const int ng = __ldcg(gd);
            if (ng <= 0) return;
            nt = NP > 0 ? min(ng, MAXT) : 1;
#pragma unroll
            for (int i = 0; i < MAXT; i++) {
                const int pe = i < nt ? __ldcg(gd + 1 + i) : 0, tk = pe >> 8, kk = pe & 255;
                xo[i] = (size_t)tk * it.xs + (size_t)kk * it.xk;
                yo[i] = (size_t)tk * it.ys + (size_t)kk * it.yk;
                if (i == 0) si = tk * it.ss + kk;
            }
        }
        const int e = __ldcg(it.sel + si);
        W = it.wtab[e];
        S = it.stab ? it.stab[e] : nullptr;
        if (it.pair) {
            W2 = it.w2tab[e];
            S2 = it.s2tab ? it.s2tab[e] : nullptr;
        }
    }
    int *kbs = reinterpret_cast<int *>(smem + kMmaRing + kMmaSRing + (size_t)nt * nb * MPU * kMmaXpPerMma);  // [nt][nb]
    double *runs = reinterpret_cast<double *>(smem + kMmaRing + kMmaSRing + (size_t)nt * nb * MPU * kMmaXpPerMma +
                                              (((size_t)nt * nb * 4 + 15) & ~(size_t)15));   // [nt][tr][8]
    // The canonical order sums eight contiguous runs of ceil(nb / 8) units;
    // R of them are non-empty. Warp w takes run w % R of row groups
    // w / R, w / R + SH, ... (SH = 8 / R warps share a run when R < 8), and
    // keeps that run's sum itself.
    const int per = (nb + 7) >> 3, R = (nb + per - 1) / per, SH = 8 / R;
    const int run = warp % R, sub = warp / R;
    const int cb0 = run * per, cb1 = min(nb, cb0 + per), ngr = it.tr >> 4;
    const int K = sub < SH ? (cb1 - cb0) * ((ngr - sub + SH - 1) / SH) : 0;   // units of this warp
    const int nsteps = K * STEPS;

    // the matrix row of virtual row v, or -1 past the matrix; *second: W2
    auto row_of = [&](int v, bool &second) -> int {
        second = it.pair && v >= trh;
        const int row = it.pair ? tile * trh + (second ? v - trh : v) : tile * it.tr + v;
        return row < it.rows ? row : -1;
    };
    // the unit walk: the warp's run in each of its row groups in turn
    int i_rg = sub, i_cb = cb0, i_s = 0, i_q = 0;
    auto issue_next = [&]() {
        if (i_q < nsteps) {
            const int slot = i_q % kMmaStages;
#pragma unroll
            for (int h = 0; h < 2; h++) {                 // rows g, g + 8
                bool second;
                const int row = row_of(i_rg * 16 + g + 8 * h, second);
                const bool ok = row >= 0;
                const uint8_t *base = (second ? W2 : W) + (size_t)(ok ? row : 0) * rb + (size_t)i_cb * UB;
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const int j = 2 * i_s + c;
                    cp_async16(&ring[(slot * 4 + h * 2 + c) * 256 + tid], ok ? base + 64 * j + 16 * t : W, ok);
                }
                if (FMT == DSV4B_WFP4 && t == 0) {        // the row's 8 scale bytes of this unit
                    const uint8_t *sb = (second ? S2 : S) + (size_t)(ok ? row : 0) * it.sc + (size_t)i_cb * 8;
                    const unsigned sa =
                        (unsigned)__cvta_generic_to_shared(&sring[((warp * kMmaStages + slot) * 8 + g) * 2 + h]);
                    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(sa), "l"(ok ? sb : S),
                                 "r"(ok ? 8 : 0) : "memory");
                }
            }
            if (++i_s == STEPS) {
                i_s = 0;
                if (++i_cb == cb1) { i_cb = cb0; i_rg += SH; }
            }
        }
        i_q++;
        cp_commit();
    };
#pragma unroll
    for (int q = 0; q < kMmaStages - 1; q++) issue_next();
    pdl_wait();

    // x fragments: every warp builds those of its own run for every token
    // (warps sharing a run write the same values); lane = (mma, t), two
    // passes for the 16 k16-steps of an FP4 unit. All of a token's x loads
    // are issued before any is used.
    constexpr int XU = kMmaMaxBlocks / 8, XH = MPU / 8;
#pragma unroll
    for (int tk = 0; tk < MAXT; tk++) {
        if (tk >= nt) break;
        const float *xt = X + xo[tk];
        uint2 *xpt = xp + tk * xtab;
        float4 xv[XU][XH];
#pragma unroll
        for (int u = 0; u < XU; u++) {
            const int cb = cb0 + u;
#pragma unroll
            for (int h = 0; h < XH; h++) {
                const int m = h * 8 + (lane >> 2), tt = lane & 3, j = m / MPC, i = m - j * MPC;
                if (cb >= cb1) {
                    xv[u][h] = make_float4(0.f, 0.f, 0.f, 0.f);
                } else if constexpr (FMT == DSV4B_WFP4) {
                    // k16 step i pairs elements (8 (i/2) + 2 (i%2) + {0, 4}) and
                    // (... + {1, 5}) of the lane's 32, as e2m1_word() pairs them
                    const float *xb = xt + cb * F::COLS + 4 * E * j + E * tt + 8 * (i >> 1) + 2 * (i & 1);
                    const float2 lo = ld_f2(xb), hi = ld_f2(xb + 4);
                    xv[u][h] = make_float4(lo.x, hi.x, lo.y, hi.y);
                } else {
                    xv[u][h] = ld_f4(xt + cb * F::COLS + 4 * E * j + E * tt + 4 * i);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < XU; u++) {
            const int cb = cb0 + u;
            if (cb >= cb1) break;
            float mx = 0.0f;
#pragma unroll
            for (int h = 0; h < XH; h++)
                mx = fmaxf(mx, fmaxf(fmaxf(fabsf(xv[u][h].x), fabsf(xv[u][h].y)),
                                     fmaxf(fabsf(xv[u][h].z), fabsf(xv[u][h].w))));
            mx = warp_max_f(mx);
            int k = 0;
            if (!BF && mx > 0.0f && mx == mx) {
                const int ex = (int)((__float_as_uint(mx) >> 23) & 0xFFu) - 127;   // floor(log2 mx), normal mx
                k = 14 - (ex < -126 ? -126 : ex);
                k = k > 126 ? 126 : (k < -126 ? -126 : k);
            }
#pragma unroll
            for (int h = 0; h < XH; h++) {
                const int m = h * 8 + (lane >> 2), tt = lane & 3;
                uint2 pc[3];
                x_pieces<BF>(xv[u][h], BF ? 1.0f : pow2f(k), pc);
#pragma unroll
                for (int p = 0; p < 3; p++) xpt[(cb * MPU + m) * 12 + tt * 3 + p] = pc[p];
            }
            if (lane == 0) kbs[tk * nb + cb] = k;
        }
    }
    __syncwarp();

    // this lane's B source: token 2 p + (g >= 3) of pair p, piece g % 3
    // (columns 6 and 7 stay zero), resolved once
    const uint2 *bsrc[NPP];
#pragma unroll
    for (int pp = 0; pp < NPP; pp++) {
        const int tk = 2 * pp + (g < 3 ? 0 : 1);
        bsrc[pp] = (g < (NP > 0 ? 6 : 3) && tk < nt) ? xp + tk * xtab + t * 3 + (g < 3 ? g : g - 3) : nullptr;
    }
    const bool two = NP > 0 && nt > 1;               // a second token in pair 0 (lanes t = 2 flush it)
    float c[NPP][4];
    double run_a[NPP], run_b[NPP];                   // lanes t = 0 / 2: rows g, g + 8 of the current row group
#pragma unroll
    for (int pp = 0; pp < NPP; pp++) {
        c[pp][0] = c[pp][1] = c[pp][2] = c[pp][3] = 0.f;
        run_a[pp] = run_b[pp] = 0.0;
    }
    int c_rg = sub, c_cb = cb0, c_s = 0;
    for (int q = 0; q < nsteps; q++) {
        issue_next();
        cp_wait<kMmaStages - 1>();
        if (FMT == DSV4B_WFP4) __syncwarp();
        const int slot = q % kMmaStages;
        // FP8 block scales of the unit's two rows, fetched before the math
        float sa = 1.0f, sbv = 1.0f;
        bool s2a = false, s2b = false;
        const int ra = row_of(c_rg * 16 + g, s2a), rbw = row_of(c_rg * 16 + g + 8, s2b);
        if (FMT == DSV4B_WFP8 && (t == 0 || (t == 2 && two)) && c_s == STEPS - 1) {
            const int col = (c_cb * F::COLS) >> it.lbc;
            sa = ra >= 0 ? e8m0(__ldg((s2a ? S2 : S) + (size_t)(ra >> it.lbr) * it.sc + col)) : 0.0f;
            sbv = rbw >= 0 ? e8m0(__ldg((s2b ? S2 : S) + (size_t)(rbw >> it.lbr) * it.sc + col)) : 0.0f;
        }
        uint4 wv[4];
#pragma unroll
        for (int r = 0; r < 4; r++) wv[r] = ring[(slot * 4 + r) * 256 + tid];
        uint32_t s4a = 0, s4b = 0;
        if (FMT == DSV4B_WFP4) {                          // scale bytes 4 j + t of rows g, g + 8
            const uint2 *sr = sring + ((warp * kMmaStages + slot) * 8 + g) * 2;
            const uint2 sp = sr[0], sq = sr[1];
            s4a = ((t < 4 ? sp.x >> (8 * t) : 0) & 0xFFu) | (((sp.y >> (8 * t)) & 0xFFu) << 8);
            s4b = ((sq.x >> (8 * t)) & 0xFFu) | (((sq.y >> (8 * t)) & 0xFFu) << 8);
        }
#pragma unroll
        for (int cc = 0; cc < 2; cc++) {
            const int j = 2 * c_s + cc;
            const uint4 &wa = wv[cc], &wb = wv[2 + cc];   // rows g, g + 8
            uint32_t ha = 0, hb = 0;
            if (FMT == DSV4B_WFP4) {
                ha = e8m0_h2x((s4a >> (8 * cc)) & 0xFFu);
                hb = e8m0_h2x((s4b >> (8 * cc)) & 0xFFu);
            }
#pragma unroll
            for (int i = 0; i < MPC; i++) {
                const int m = j * MPC + i;
                // the weights' A fragments, formed once for every token pair
                uint32_t a0, a1, a2, a3;
                if constexpr (FMT == DSV4B_WFP8) {
                    const uint32_t va = word_of(wa, i), vb = word_of(wb, i);
                    a0 = e4m3x2_h2(va);
                    a1 = e4m3x2_h2(vb);
                    a2 = e4m3x2_h2(va >> 16);
                    a3 = e4m3x2_h2(vb >> 16);
                } else if constexpr (FMT == DSV4B_WFP4) {
                    // word i/2 of each row (decoded once for both of its
                    // steps); step i takes nibble pairs (2 (i%2), +4) and
                    // (2 (i%2) + 1, +4)
                    uint32_t ra4[4], rb4[4];
                    e2m1_word(word_of(wa, i >> 1), ra4);
                    e2m1_word(word_of(wb, i >> 1), rb4);
                    const int q0 = 2 * (i & 1);
                    a0 = hmul2(ra4[q0], ha);
                    a1 = hmul2(rb4[q0], hb);
                    a2 = hmul2(ra4[q0 + 1], ha);
                    a3 = hmul2(rb4[q0 + 1], hb);
                } else {
                    a0 = word_of(wa, 2 * i);
                    a1 = word_of(wb, 2 * i);
                    a2 = word_of(wa, 2 * i + 1);
                    a3 = word_of(wb, 2 * i + 1);
                }
                const int xo = (c_cb * MPU + m) * 12;
#pragma unroll
                for (int pp = 0; pp < NPP; pp++) {
                    uint2 b = make_uint2(0u, 0u);
                    if (bsrc[pp]) b = bsrc[pp][xo];
                    if constexpr (BF) mma_bf16(c[pp], a0, a1, a2, a3, b.x, b.y);
                    else mma_f16(c[pp], a0, a1, a2, a3, b.x, b.y);
                }
            }
        }
        if (FMT == DSV4B_WFP4) __syncwarp();
        if (c_s == STEPS - 1) {
            // flush the unit: token A's pieces (n = 0, 1, 2) sit on lanes t = 0
            // (n = 0, 1) and t = 1 (n = 2); token B's (n = 3, 4, 5) on t = 1
            // (n = 3) and t = 2 (n = 4, 5); rows g (c0, c1) and g + 8 (c2, c3)
#pragma unroll
            for (int pp = 0; pp < NPP; pp++) {
                const float n2a = __shfl_sync(0xffffffffu, c[pp][0], lane | 1);
                const float n2b = __shfl_sync(0xffffffffu, c[pp][2], lane | 1);
                float n3a = 0.f, n3b = 0.f;
                if (two) {                                // warp-uniform
                    n3a = __shfl_sync(0xffffffffu, c[pp][1], (lane & ~3) | 1);
                    n3b = __shfl_sync(0xffffffffu, c[pp][3], (lane & ~3) | 1);
                }
                const int tk = 2 * pp + (t == 2 ? 1 : 0);
                if ((t == 0 || (NP > 0 && t == 2)) && tk < nt) {
                    const float un = pow2f(-kbs[tk * nb + c_cb]);
                    const float pa = t == 0 ? __fadd_rn(__fadd_rn(c[pp][0], c[pp][1]), n2a)
                                            : __fadd_rn(__fadd_rn(n3a, c[pp][0]), c[pp][1]);
                    const float pb = t == 0 ? __fadd_rn(__fadd_rn(c[pp][2], c[pp][3]), n2b)
                                            : __fadd_rn(__fadd_rn(n3b, c[pp][2]), c[pp][3]);
                    const float qa = __fmul_rn(__fmul_rn(pa, un), sa);
                    const float qb = __fmul_rn(__fmul_rn(pb, un), sbv);
                    run_a[pp] = __dadd_rn(run_a[pp], (double)qa);
                    run_b[pp] = __dadd_rn(run_b[pp], (double)qb);
                    if (c_cb == cb1 - 1) {                // the run ends: its sums are final
                        double *rt = runs + (size_t)tk * it.tr * 8;
                        rt[(c_rg * 16 + g) * 8 + run] = run_a[pp];
                        rt[(c_rg * 16 + g + 8) * 8 + run] = run_b[pp];
                        run_a[pp] = run_b[pp] = 0.0;
                    }
                }
                c[pp][0] = c[pp][1] = c[pp][2] = c[pp][3] = 0.f;
            }
        }
        if (++c_s == STEPS) {
            c_s = 0;
            if (++c_cb == cb1) { c_cb = cb0; c_rg += SH; }
        }
    }
    cp_wait<0>();
    __syncthreads();
    // row totals: the eight run sums of a virtual row added in run order
    // (an empty run adds 0), per token
    auto total = [&](int tk, int v) {
        const double *rt = runs + (size_t)tk * it.tr * 8;
        double tt = 0.0;
#pragma unroll
        for (int w = 0; w < 8; w++) tt = __dadd_rn(tt, w < R ? rt[v * 8 + w] : 0.0);
        return (float)tt;
    };
    const int nreal = it.pair ? trh : it.tr;
#pragma unroll
    for (int tk = 0; tk < MAXT; tk++) {
        if (tk >= nt) break;
        float *yt = Y + yo[tk];
        for (int r = tid; r < nreal; r += blockDim.x) {
            const int row = tile * nreal + r;
            if (row >= it.rows) break;
            float a = total(tk, r);
            if (it.pair) a = swiglu_pair(a, total(tk, r + trh), it.limit);
            yt[row] = a;
        }
    }
}

}  // namespace dsv4b

// gemv_core.cuh - the one summation order every GEMV kernel in this backend
// uses, so results never depend on which kernel, grid or batch size ran.
//
// A row is cut into SEGMENTS of 256 weight bytes (64 f32 / 128 bf16 / 256 fp8
// / 512 fp4 elements), each owned by 16 lanes. Lane li (0..15) of a segment
// takes NSTEP steps (1 / 2 / 4 / 8); step k covers the 4 elements
// [4(16k+li), 4(16k+li)+4) of the segment, so at every step the 16 lanes read
// 16 consecutive float4 of x (bank-conflict-free in shared memory) and
// consecutive weight bytes. For row o, token t, lane li:
//   c     = a float2 accumulator: per step, fma of elements (0,1) then (2,3)
//           into (c.x, c.y);
//   q     = at the lane's last step inside each scale block (every step for
//           unscaled formats ends the single block at the lane's last step):
//           q = fma(c.x + c.y, scale, q) and c restarts at 0 (the scale is a
//           power of two, so the product is exact);
//   seg   = the 16 lanes' q summed in float by the xor butterfly 8,4,2,1;
//   total = ((0 + seg_0) + seg_1) + ...   in DOUBLE, in segment order;
//   y     = (float)total.
// Missing elements of a short last segment contribute nothing. Block sizes are
// powers of two. Against the reference CPU's 16-lane double tree
// (src/core/dsv4_matmul.c:51-64) this agrees to ~1e-7 of the vector scale;
// between kernels of this backend it is bit-identical, which is what makes
// mmq_n equal nt separate mmq calls.
#pragma once

#include "common.cuh"

namespace dsv4b {

template <int FMT> struct Fmt;
// NSTEP: steps per lane per segment; SB: weight bytes per step; EPU kept for
// element <-> byte arithmetic (elements per 16 weight bytes).
template <> struct Fmt<DSV4B_WF32> { static constexpr int NSTEP = 1, SB = 16, EPU = 4; static constexpr bool SC = false; };
template <> struct Fmt<DSV4B_WBF16> { static constexpr int NSTEP = 2, SB = 8, EPU = 8; static constexpr bool SC = false; };
template <> struct Fmt<DSV4B_WFP8> { static constexpr int NSTEP = 4, SB = 4, EPU = 16; static constexpr bool SC = true; };
template <> struct Fmt<DSV4B_WFP4> { static constexpr int NSTEP = 8, SB = 2, EPU = 32; static constexpr bool SC = true; };

// The raw weight bytes of one step, widened to 16 bytes (unused words 0).
template <int FMT>
__device__ __forceinline__ uint4 load_step(const uint8_t *p)
{
    if constexpr (FMT == DSV4B_WF32) return *reinterpret_cast<const uint4 *>(p);
    else if constexpr (FMT == DSV4B_WBF16) {
        const uint2 v = *reinterpret_cast<const uint2 *>(p);
        return make_uint4(v.x, v.y, 0u, 0u);
    } else if constexpr (FMT == DSV4B_WFP8) return make_uint4(*reinterpret_cast<const uint32_t *>(p), 0u, 0u, 0u);
    else return make_uint4((uint32_t)*reinterpret_cast<const uint16_t *>(p), 0u, 0u, 0u);
}

// Streaming (L1 no-allocate) global form of load_step, for weights read once.
template <int FMT>
__device__ __forceinline__ uint4 ldg_step(const uint8_t *p)
{
    uint4 r = make_uint4(0u, 0u, 0u, 0u);
    if constexpr (FMT == DSV4B_WF32)
        asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    else if constexpr (FMT == DSV4B_WBF16)
        asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    else if constexpr (FMT == DSV4B_WFP8)
        asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r.x) : "l"(p));
    else {
        unsigned short h;
        asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(h) : "l"(p));
        r.x = h;
    }
    return r;
}

// Two float pairs of one step's 4 weights.
template <int FMT>
__device__ __forceinline__ void step_decode(const uint4 &w, float2 &a, float2 &b)
{
    if constexpr (FMT == DSV4B_WF32) {
        a = make_float2(__uint_as_float(w.x), __uint_as_float(w.y));
        b = make_float2(__uint_as_float(w.z), __uint_as_float(w.w));
    } else if constexpr (FMT == DSV4B_WBF16) {
        a = bf16x2(w.x);
        b = bf16x2(w.y);
    } else if constexpr (FMT == DSV4B_WFP8) {
        a = e4m3x2((uint16_t)(w.x & 0xFFFFu));
        b = e4m3x2((uint16_t)(w.x >> 16));
    } else {
        a = e2m1x2((uint8_t)(w.x & 0xFFu));
        b = e2m1x2((uint8_t)((w.x >> 8) & 0xFFu));
    }
}

// Which of a lane's NS steps exist (a prefix) and which of them close a scale
// block, for the segment starting at row element `e0` (power-of-two blocks of
// 2^lbc elements; unscaled formats pass a huge lbc). `nvalid` = valid steps.
struct StepMasks {
    uint32_t flush;
    int nvalid;
};
template <int FMT>
__device__ __forceinline__ StepMasks step_masks(int e0, int li, int nvalid, int lbc)
{
    constexpr int NS = Fmt<FMT>::NSTEP;
    StepMasks m;
    m.nvalid = nvalid;
    m.flush = 0u;
#pragma unroll
    for (int k = 0; k < NS; k++) {
        const int ek = e0 + 4 * (16 * k + li), en = e0 + 4 * (16 * (k + 1) + li);
        if (k < nvalid && (k + 1 == nvalid || (ek >> lbc) != (en >> lbc))) m.flush |= 1u << k;
    }
    return m;
}

// q of one lane for one row and token (see the order above). w[k], x[k] are
// the step's weights and x; s[k] the scale of step k's block.
template <int FMT>
__device__ __forceinline__ float lane_q(const uint4 *w, const float4 *x, const float *s, const StepMasks &m)
{
    constexpr int NS = Fmt<FMT>::NSTEP;
    float q = 0.0f;
    float2 c = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < NS; k++) {
        if (k < m.nvalid) {
            float2 a, b;
            step_decode<FMT>(w[k], a, b);
            c = fma2(a, make_float2(x[k].x, x[k].y), c);
            c = fma2(b, make_float2(x[k].z, x[k].w), c);
            if (m.flush & (1u << k)) {
                q = __fmaf_rn(__fadd_rn(c.x, c.y), s[k], q);
                c = make_float2(0.f, 0.f);
            }
        }
    }
    return q;
}

// The segment sum: xor butterfly over the 16 lanes of a half-warp. Every lane
// of the warp must call it (full-mask shuffles); offsets < 16 keep each half
// separate, and every lane of a half ends with the same bits.
__device__ __forceinline__ float seg_sum16(float v)
{
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace dsv4b

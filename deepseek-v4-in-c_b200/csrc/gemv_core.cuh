// gemv_core.cuh - the one summation order every GEMV kernel in this backend
// uses, so results never depend on which kernel, grid or batch size ran.
//
// Row o, token t, weights in 16-byte UNITS (4 f32 / 8 bf16 / 16 fp8 / 32 fp4
// elements; a unit never straddles a scale block):
//   p_u  = two float chains over the unit (even / odd elements, fma in element
//          order), then p_u = even + odd;
//   q_u  = p_u * scale_u            (exact: the scale is a power of two);
//   seg_j = the 16 q_u of units [16j, 16j+16) summed in float by the xor
//          butterfly 8,4,2,1 (missing units of a short last segment are 0);
//   total = ((0 + seg_0) + seg_1) + ...   in DOUBLE, in segment order;
//   y     = (float)total.
// Against the reference CPU's 16-lane double tree (src/core/dsv4_matmul.c:
// 51-64) this agrees to ~1e-7 of the vector scale; between kernels of this
// backend it is bit-identical, which is what makes mmq_n equal nt mmq calls.
#pragma once

#include "common.cuh"

namespace dsv4b {

template <int FMT> struct Fmt;
template <> struct Fmt<DSV4B_WF32> { static constexpr int EPU = 4; static constexpr bool SC = false; };
template <> struct Fmt<DSV4B_WBF16> { static constexpr int EPU = 8; static constexpr bool SC = false; };
template <> struct Fmt<DSV4B_WFP8> { static constexpr int EPU = 16; static constexpr bool SC = true; };
template <> struct Fmt<DSV4B_WFP4> { static constexpr int EPU = 32; static constexpr bool SC = true; };

// Decode elements [4k, 4k+4) of a unit into two float pairs.
template <int FMT>
__device__ __forceinline__ void decode4(const uint4 &u, int k, float2 &a, float2 &b)
{
    const uint32_t w0 = (k == 0) ? u.x : (k == 1) ? u.y : (k == 2) ? u.z : u.w;
    if constexpr (FMT == DSV4B_WF32) {
        a = make_float2(__uint_as_float(u.x), __uint_as_float(u.y));
        b = make_float2(__uint_as_float(u.z), __uint_as_float(u.w));
    } else if constexpr (FMT == DSV4B_WBF16) {
        const uint32_t lo = (k == 0) ? u.x : u.z, hi = (k == 0) ? u.y : u.w;
        a = bf16x2(lo);
        b = bf16x2(hi);
    } else if constexpr (FMT == DSV4B_WFP8) {
        a = e4m3x2((uint16_t)(w0 & 0xFFFFu));
        b = e4m3x2((uint16_t)(w0 >> 16));
    } else {
        const uint32_t w = (k < 2) ? ((k == 0) ? u.x : u.x >> 16)
                         : (k < 4) ? ((k == 2) ? u.y : u.y >> 16)
                         : (k < 6) ? ((k == 4) ? u.z : u.z >> 16)
                                   : ((k == 6) ? u.w : u.w >> 16);
        a = e2m1x2((uint8_t)(w & 0xFFu));
        b = e2m1x2((uint8_t)((w >> 8) & 0xFFu));
    }
}

// p_u for one unit against EPU floats of x (x 16-byte aligned).
template <int FMT>
__device__ __forceinline__ float unit_dot(const uint4 &w, const float *x)
{
    constexpr int EPU = Fmt<FMT>::EPU;
    float2 c = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < EPU / 4; k++) {
        const float4 xv = *reinterpret_cast<const float4 *>(x + 4 * k);
        float2 a, b;
        decode4<FMT>(w, k, a, b);
        c = fma2(a, make_float2(xv.x, xv.y), c);
        c = fma2(b, make_float2(xv.z, xv.w), c);
    }
    return __fadd_rn(c.x, c.y);
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

// gemv_core.cuh - the one summation order every GEMV kernel in this backend
// uses, so a result never depends on which kernel, grid or batch size ran.
//
// A row is cut into SEGMENTS of 256 weight bytes (64 f32 / 128 bf16 / 256 fp8
// / 512 fp4 elements), each owned by 16 lanes. Lane li (0..15) owns the 16
// contiguous bytes [16 li, 16 li + 16) of its segment -- E = 4 / 8 / 16 / 32
// elements, one 128-bit load -- and walks them in NS = E / 4 sub-steps of 4
// elements. For row o, token t, lane li:
//   c     = a float2 accumulator: per sub-step, fma of elements (0,1) then
//           (2,3) into (c.x, c.y);
//   q     = at the lane's last sub-step inside each scale block (for unscaled
//           formats: at its last sub-step): q = fma(c.x + c.y, scale, q), and
//           c restarts at 0 (scales are powers of two, so the product is
//           exact);
//   seg   = the 16 lanes' q summed in float by the xor butterfly 8,4,2,1;
//   total = ((0 + seg_0) + seg_1) + ...   in DOUBLE, in segment order;
//   y     = (float)total.
// Lanes past the end of a short last segment contribute 0. Against the
// reference CPU's 16-lane double tree (src/core/dsv4_matmul.c:51-64) this
// agrees to ~1e-7 of the vector scale; between kernels of this backend it is
// bit-identical, which is what makes mmq_n equal nt separate mmq calls.
#pragma once

#include "common.cuh"

namespace dsv4b {

// E: elements per lane (16 bytes); NS: 4-element sub-steps; LE: log2(E).
template <int FMT> struct Fmt;
template <> struct Fmt<DSV4B_WF32> { static constexpr int E = 4, NS = 1, LE = 2; static constexpr bool SC = false; };
template <> struct Fmt<DSV4B_WBF16> { static constexpr int E = 8, NS = 2, LE = 3; static constexpr bool SC = false; };
template <> struct Fmt<DSV4B_WFP8> { static constexpr int E = 16, NS = 4, LE = 4; static constexpr bool SC = true; };
template <> struct Fmt<DSV4B_WFP4> { static constexpr int E = 32, NS = 8, LE = 5; static constexpr bool SC = true; };

__device__ __forceinline__ uint32_t word_of(const uint4 &w, int i)
{
    return i == 0 ? w.x : i == 1 ? w.y : i == 2 ? w.z : w.w;
}

// The 4 weights of sub-step K of a lane's 16 bytes, as two float pairs.
template <int FMT, int K>
__device__ __forceinline__ void sub_decode(const uint4 &w, float2 &a, float2 &b)
{
    if constexpr (FMT == DSV4B_WF32) {
        a = make_float2(__uint_as_float(w.x), __uint_as_float(w.y));
        b = make_float2(__uint_as_float(w.z), __uint_as_float(w.w));
    } else if constexpr (FMT == DSV4B_WBF16) {
        a = bf16x2(word_of(w, 2 * K));
        b = bf16x2(word_of(w, 2 * K + 1));
    } else if constexpr (FMT == DSV4B_WFP8) {
        const uint32_t v = word_of(w, K);
        a = e4m3x2((uint16_t)(v & 0xFFFFu));
        b = e4m3x2((uint16_t)(v >> 16));
    } else {
        const uint32_t v = word_of(w, K >> 1);
        const uint32_t h = (K & 1) ? (v >> 16) : (v & 0xFFFFu);
        a = e2m1x2((uint8_t)(h & 0xFFu));
        b = e2m1x2((uint8_t)(h >> 8));
    }
}

// Which sub-steps close a scale block, for a lane whose first element is e
// (row element index) in blocks of 2^lbc elements; unscaled formats pass a
// huge lbc, so only the last sub-step flushes.
template <int FMT>
__device__ __forceinline__ uint32_t flush_mask(int e, int lbc)
{
    constexpr int NS = Fmt<FMT>::NS;
    uint32_t m = 1u << (NS - 1);
#pragma unroll
    for (int k = 0; k + 1 < NS; k++)
        if (((e + 4 * k) >> lbc) != ((e + 4 * k + 4) >> lbc)) m |= 1u << k;
    return m;
}

// q of one lane for one row and token (the order above). x[k] is sub-step
// k's float4 of x; s[k] the scale of sub-step k's block.
template <int FMT>
__device__ __forceinline__ float lane_q(const uint4 &w, const float4 *x, const float *s, uint32_t flush)
{
    float q = 0.0f;
    float2 c = make_float2(0.f, 0.f);
    float2 a, b;
#define DSV4B_SUB(K)                                                                \
    if constexpr ((K) < Fmt<FMT>::NS) {                                             \
        sub_decode<FMT, (K)>(w, a, b);                                              \
        c = fma2(a, make_float2(x[K].x, x[K].y), c);                                \
        c = fma2(b, make_float2(x[K].z, x[K].w), c);                                \
        if (flush & (1u << (K))) {                                                  \
            q = __fmaf_rn(__fadd_rn(c.x, c.y), s[K], q);                            \
            c = make_float2(0.f, 0.f);                                              \
        }                                                                           \
    }
    DSV4B_SUB(0) DSV4B_SUB(1) DSV4B_SUB(2) DSV4B_SUB(3)
    DSV4B_SUB(4) DSV4B_SUB(5) DSV4B_SUB(6) DSV4B_SUB(7)
#undef DSV4B_SUB
    return q;
}

// The segment sum: xor butterfly over the 16 lanes of a half-warp. `mask`
// names the calling half-warp's lanes (offsets < 16 never leave it), so the
// two halves of a warp may run different code.
__device__ __forceinline__ float seg_sum16(float v, unsigned mask)
{
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(mask, v, o));
    return v;
}

__device__ __forceinline__ unsigned half_mask() { return 0xFFFFu << (threadIdx.x & 16); }

}  // namespace dsv4b

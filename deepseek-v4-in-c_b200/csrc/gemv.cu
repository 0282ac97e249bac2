// gemv.cu - block-scaled GEMV / skinny GEMM against HBM-resident weights.
//
// Replaces the reference's k_mmq_fp8 / k_mmq_fp8_n (src/cuda/dsv4_cuda.cu:93-230)
// and widens it to the four storage formats dsv4_mmq dispatches on
// (src/core/dsv4_matmul.c:516-591): FP8 128x128, FP4 1x32, BF16 and F32.
//
// Batch-1 decode is HBM-bound (one multiply-add per weight byte for FP8), so
// the kernel is a weight stream: every lane issues 16-byte non-allocating loads,
// several rows x several units deep, decodes in registers with the hardware
// e4m3/e2m1 converters and multiplies with packed f32x2 FMAs. x is read through
// L1 (it is shared by every row) and each x chunk is reused by R rows.
//
// ARITHMETIC (fixed, independent of R, NT and the grid):
//   a 16-byte unit of one row holds EPU elements (4 f32, 8 bf16, 16 fp8,
//   32 fp4) that never straddle a scale block. Its dot product is two float
//   chains (even / odd elements, fma in element order), summed, multiplied by
//   the block scale (exact: a power of two), and added into a per-lane DOUBLE.
//   Lanes take units lane, lane+32, ...; the 32 lane totals are folded by a
//   fixed xor butterfly in double and rounded to float once.
// The reduction of one (row, token) therefore never depends on how many rows or
// tokens share the launch, which makes mmq_n bit-identical to nt separate mmq
// calls -- the property the reference's GPU gate checks
// (tests/unit/test_cuda.c:194-257). Against the reference CPU's double tree it
// agrees to ~1e-7 relative.
#include "common.cuh"
#include "internal.h"

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
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    if constexpr (FMT == DSV4B_WF32) {
        a = make_float2(__uint_as_float(w[0]), __uint_as_float(w[1]));
        b = make_float2(__uint_as_float(w[2]), __uint_as_float(w[3]));
    } else if constexpr (FMT == DSV4B_WBF16) {
        a = bf16x2(w[2 * k]);
        b = bf16x2(w[2 * k + 1]);
    } else if constexpr (FMT == DSV4B_WFP8) {
        a = e4m3x2((uint16_t)(w[k] & 0xFFFFu));
        b = e4m3x2((uint16_t)(w[k] >> 16));
    } else {
        const uint32_t h = w[k >> 1] >> ((k & 1) * 16);
        a = e2m1x2((uint8_t)(h & 0xFFu));
        b = e2m1x2((uint8_t)((h >> 8) & 0xFFu));
    }
}

template <int FMT, int NT, int R, int U>
__global__ void __launch_bounds__(64)
k_gemv(GemvArgs g)
{
    constexpr int EPU = Fmt<FMT>::EPU;
    const int lane = threadIdx.x & 31;
    const int warp = (int)((blockIdx.x * (unsigned)blockDim.x + threadIdx.x) >> 5);
    const int row0 = warp * R;
    if (row0 >= g.rows) return;
    const int upr = g.rowbytes >> 4;

    const uint8_t *wr[R];
    int srow[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
        const int o = min(row0 + r, g.rows - 1);
        wr[r] = g.W + (size_t)o * g.rowbytes;
        srow[r] = (o / g.blk_r) * g.sc;
    }

    double acc[R][NT];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int t = 0; t < NT; t++) acc[r][t] = 0.0;

    for (int u0 = lane; u0 < upr; u0 += 32 * U) {
        uint4 wv[U][R];
#pragma unroll
        for (int j = 0; j < U; j++) {
            const int u = u0 + 32 * j;
#pragma unroll
            for (int r = 0; r < R; r++)
                if (u < upr) wv[j][r] = ld_stream16(wr[r] + (size_t)u * 16);
        }
#pragma unroll
        for (int j = 0; j < U; j++) {
            const int u = u0 + 32 * j;
            if (u < upr) {
                const int col0 = u * EPU;
                float2 c[R][NT];
#pragma unroll
                for (int r = 0; r < R; r++)
#pragma unroll
                    for (int t = 0; t < NT; t++) c[r][t] = make_float2(0.f, 0.f);
#pragma unroll
                for (int k = 0; k < EPU / 4; k++) {
                    float4 xv[NT];
#pragma unroll
                    for (int t = 0; t < NT; t++)
                        xv[t] = ld_f4(g.x + (size_t)t * g.xstride + col0 + 4 * k);
#pragma unroll
                    for (int r = 0; r < R; r++) {
                        float2 wa, wb;
                        decode4<FMT>(wv[j][r], k, wa, wb);
#pragma unroll
                        for (int t = 0; t < NT; t++) {
                            c[r][t] = fma2(wa, make_float2(xv[t].x, xv[t].y), c[r][t]);
                            c[r][t] = fma2(wb, make_float2(xv[t].z, xv[t].w), c[r][t]);
                        }
                    }
                }
#pragma unroll
                for (int r = 0; r < R; r++) {
                    double s = 1.0;
                    if constexpr (Fmt<FMT>::SC) s = (double)e8m0(g.S[srow[r] + col0 / g.blk_c]);
#pragma unroll
                    for (int t = 0; t < NT; t++) {
                        const float p = __fadd_rn(c[r][t].x, c[r][t].y);
                        acc[r][t] = __fma_rn((double)p, s, acc[r][t]);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int t = 0; t < NT; t++) {
            const double v = warp_sum_d(acc[r][t]);
            if (lane == 0 && row0 + r < g.rows)
                g.y[(size_t)t * g.ystride + row0 + r] = (float)v;
        }
}

// Any shape: one warp per (row, token), scalar loads, exact products summed in
// double. Only reached by shapes whose rows are not 16-byte multiples (the
// reference's hand-sized test matrices); every model matrix takes k_gemv.
__global__ void k_gemv_generic(GemvArgs g, int fmt, int nt)
{
    const int lane = threadIdx.x & 31;
    const long warp = (long)((blockIdx.x * (unsigned)blockDim.x + threadIdx.x) >> 5);
    if (warp >= (long)g.rows * nt) return;
    const int o = (int)(warp % g.rows), t = (int)(warp / g.rows);
    const float *x = g.x + (size_t)t * g.xstride;
    const uint8_t *row = g.W + (size_t)o * g.rowbytes;
    double acc = 0.0;
    for (int c = lane; c < g.cols; c += 32) {
        float w;
        if (fmt == DSV4B_WF32) w = reinterpret_cast<const float *>(row)[c];
        else if (fmt == DSV4B_WBF16) w = __uint_as_float((uint32_t)reinterpret_cast<const uint16_t *>(row)[c] << 16);
        else if (fmt == DSV4B_WFP8) w = e4m3x2((uint16_t)row[c]).x;
        else { const uint8_t b = row[c >> 1]; w = e2m1x2((uint8_t)((c & 1) ? (b >> 4) : (b & 15))).x; }
        double s = 1.0;
        if (fmt >= DSV4B_WFP8) s = (double)e8m0(g.S[(o / g.blk_r) * g.sc + c / g.blk_c]);
        acc = __fma_rn((double)w * s, (double)x[c], acc);
    }
    acc = warp_sum_d(acc);
    if (lane == 0) g.y[(size_t)t * g.ystride + o] = (float)acc;
}

template <int FMT, int NT>
static void launch_nt(const GemvArgs &g, cudaStream_t st)
{
    constexpr int R = (NT <= 2) ? 4 : (NT <= 4 ? 2 : 1);
    constexpr int U = (NT <= 4) ? 4 : 2;
    const int warps = (g.rows + R - 1) / R;
    const int threads = 64;
    const int blocks = (warps * 32 + threads - 1) / threads;
    k_gemv<FMT, NT, R, U><<<blocks, threads, 0, st>>>(g);
}

template <int FMT>
static void launch_fmt(const GemvArgs &g, int nt, cudaStream_t st)
{
    switch (nt) {
    case 1: launch_nt<FMT, 1>(g, st); break;
    case 2: launch_nt<FMT, 2>(g, st); break;
    case 3: launch_nt<FMT, 3>(g, st); break;
    case 4: launch_nt<FMT, 4>(g, st); break;
    case 5: launch_nt<FMT, 5>(g, st); break;
    case 6: launch_nt<FMT, 6>(g, st); break;
    case 7: launch_nt<FMT, 7>(g, st); break;
    default: launch_nt<FMT, 8>(g, st); break;
    }
}

static int epu_of(int fmt)
{
    return fmt == DSV4B_WF32 ? 4 : fmt == DSV4B_WBF16 ? 8 : fmt == DSV4B_WFP8 ? 16 : 32;
}

size_t row_bytes(int fmt, int cols)
{
    switch (fmt) {
    case DSV4B_WF32: return (size_t)cols * 4;
    case DSV4B_WBF16: return (size_t)cols * 2;
    case DSV4B_WFP8: return (size_t)cols;
    default: return (size_t)cols / 2;
    }
}

bool gemv_vectorizable(int fmt, const void *W, int cols, int blk_c, const float *x, long xstride)
{
    const size_t rb = row_bytes(fmt, cols);
    if (rb % 16 || ((uintptr_t)W & 15) || ((uintptr_t)x & 15) || (xstride & 3)) return false;
    if (fmt >= DSV4B_WFP8 && (blk_c <= 0 || blk_c % epu_of(fmt))) return false;
    return true;
}

int gemv(int fmt, float *y, long ystride, const float *x, long xstride,
         const void *W, const uint8_t *S, int rows, int cols, int blk_r,
         int blk_c, int nt, cudaStream_t st)
{
    if (rows <= 0 || cols <= 0 || nt <= 0) return 0;
    if (fmt == DSV4B_WFP4 && (cols & 1)) return -1;
    GemvArgs g;
    g.W = (const uint8_t *)W; g.S = S;
    g.rows = rows; g.cols = cols;
    g.blk_r = blk_r > 0 ? blk_r : 1; g.blk_c = blk_c > 0 ? blk_c : 1;
    g.sc = fmt >= DSV4B_WFP8 ? (cols + g.blk_c - 1) / g.blk_c : 0;
    g.rowbytes = (int)row_bytes(fmt, cols);
    g.xstride = xstride; g.ystride = ystride;
    if (!gemv_vectorizable(fmt, W, cols, blk_c, x, xstride)) {
        g.x = x; g.y = y;
        const long warps = (long)rows * nt;
        k_gemv_generic<<<(unsigned)((warps * 32 + 127) / 128), 128, 0, st>>>(g, fmt, nt);
        return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
    }
    for (int t0 = 0; t0 < nt; t0 += 8) {
        const int n = (nt - t0 < 8) ? nt - t0 : 8;
        g.x = x + (size_t)t0 * xstride;
        g.y = y + (size_t)t0 * ystride;
        switch (fmt) {
        case DSV4B_WF32: launch_fmt<DSV4B_WF32>(g, n, st); break;
        case DSV4B_WBF16: launch_fmt<DSV4B_WBF16>(g, n, st); break;
        case DSV4B_WFP8: launch_fmt<DSV4B_WFP8>(g, n, st); break;
        default: launch_fmt<DSV4B_WFP4>(g, n, st); break;
        }
    }
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

// Device decoder dump for the all-codes gate (reference dsv4_cuda.cu:454-469).
__global__ void k_dump_e4m3(float *out)
{
    const int i = threadIdx.x;
    if (i < 256) out[i] = e4m3x2((uint16_t)i).x;
}

int dump_e4m3(float *dev_out, cudaStream_t st)
{
    k_dump_e4m3<<<1, 256, 0, st>>>(dev_out);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace dsv4b

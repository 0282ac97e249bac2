// gemv.cu - GEMV / skinny GEMM against HBM-resident weights: the register
// kernel (batched tokens, and shapes the TMA pipeline does not take), the
// generic any-shape kernel, and the dispatch.
//
// Replaces the reference's k_mmq_fp8 / k_mmq_fp8_n (src/cuda/dsv4_cuda.cu:93-230)
// and widens it to the four storage formats dsv4_mmq dispatches on
// (src/core/dsv4_matmul.c:516-591): FP8 128x128, FP4 1x32, BF16 and F32.
// Batch-1 calls go to the TMA pipeline in gemv_tma.cu; every kernel sums in
// the order fixed by gemv_core.cuh, so a token's result never depends on the
// kernel, the grid or the batch it ran in.
#include "gemv_core.cuh"
#include "internal.h"

namespace dsv4b {

// One warp: R rows x NT tokens. Half-warp h takes segments j = h, h+2, ...;
// lane (l & 15) takes unit 16j + (l & 15). Segment sums fold into lane 0's
// double totals in segment order (seg 2m from half 0, then 2m+1 from half 1).
template <int FMT, int NT, int R, int UP>
__global__ void __launch_bounds__(64)
k_gemv_reg(GemvArgs g)
{
    constexpr int EPU = Fmt<FMT>::EPU;
    const int lane = threadIdx.x & 31, half = lane >> 4, li = lane & 15;
    const int warp = (int)((blockIdx.x * (unsigned)blockDim.x + threadIdx.x) >> 5);
    const int row0 = warp * R;
    if (row0 >= g.rows) return;
    const int upr = g.rowbytes >> 4, nseg = (upr + 15) >> 4;

    const uint8_t *wr[R];
    int srow[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
        const int o = min(row0 + r, g.rows - 1);
        wr[r] = g.W + (size_t)o * g.rowbytes;
        srow[r] = Fmt<FMT>::SC ? ((FMT == DSV4B_WFP4) ? o * g.sc : (o / g.blk_r) * g.sc) : 0;
    }
    double tot[R][NT];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int t = 0; t < NT; t++) tot[r][t] = 0.0;

    for (int m0 = 0; m0 < nseg; m0 += 2 * UP) {
        uint4 wv[UP][R];
#pragma unroll
        for (int j = 0; j < UP; j++) {
            const int seg = m0 + 2 * j + half, u = seg * 16 + li;
#pragma unroll
            for (int r = 0; r < R; r++)
                if (seg < nseg && u < upr) wv[j][r] = ld_stream16(wr[r] + (size_t)u * 16);
        }
#pragma unroll
        for (int j = 0; j < UP; j++) {
            const int seg = m0 + 2 * j + half, u = seg * 16 + li;
            const bool ok = (seg < nseg && u < upr);
            float q[R][NT];
#pragma unroll
            for (int r = 0; r < R; r++) {
                float s = 1.0f;
                if constexpr (Fmt<FMT>::SC) {
                    if (ok) s = e8m0(__ldg(g.S + srow[r] + (u * EPU) / g.blk_c));
                }
#pragma unroll
                for (int t = 0; t < NT; t++)
                    q[r][t] = ok ? __fmul_rn(unit_dot<FMT>(wv[j][r], g.x + (size_t)t * g.xstride + (size_t)u * EPU), s)
                                 : 0.0f;
            }
            const int sev = m0 + 2 * j;
#pragma unroll
            for (int r = 0; r < R; r++)
#pragma unroll
                for (int t = 0; t < NT; t++) {
                    const float v = seg_sum16(q[r][t]);
                    const float vodd = __shfl_sync(0xffffffffu, v, 16);
                    if (lane == 0) {
                        if (sev < nseg) tot[r][t] = __dadd_rn(tot[r][t], (double)v);
                        if (sev + 1 < nseg) tot[r][t] = __dadd_rn(tot[r][t], (double)vodd);
                    }
                }
        }
    }
    if (lane == 0)
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
            for (int t = 0; t < NT; t++)
                if (row0 + r < g.rows) g.y[(size_t)t * g.ystride + row0 + r] = (float)tot[r][t];
}

// Any shape: one warp per (row, token), scalar loads, exact products summed in
// double. Only reached by shapes whose rows are not 16-byte multiples (the
// reference's hand-sized test matrices); every model matrix takes the others.
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
    constexpr int R = (NT <= 2) ? 2 : 1;
    constexpr int UP = (NT <= 2) ? 2 : 1;
    const int warps = (g.rows + R - 1) / R;
    const int threads = 64;
    const int blocks = (warps * 32 + threads - 1) / threads;
    k_gemv_reg<FMT, NT, R, UP><<<blocks, threads, 0, st>>>(g);
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

int gemv_reg(const GemvArgs &g0, int fmt, int nt, cudaStream_t st)
{
    GemvArgs g = g0;
    for (int t0 = 0; t0 < nt; t0 += 8) {
        const int n = (nt - t0 < 8) ? nt - t0 : 8;
        g.x = g0.x + (size_t)t0 * g0.xstride;
        g.y = g0.y + (size_t)t0 * g0.ystride;
        switch (fmt) {
        case DSV4B_WF32: launch_fmt<DSV4B_WF32>(g, n, st); break;
        case DSV4B_WBF16: launch_fmt<DSV4B_WBF16>(g, n, st); break;
        case DSV4B_WFP8: launch_fmt<DSV4B_WFP8>(g, n, st); break;
        default: launch_fmt<DSV4B_WFP4>(g, n, st); break;
        }
    }
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
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
    g.x = x; g.y = y;
    if (!gemv_vectorizable(fmt, W, cols, blk_c, x, xstride)) {
        const long warps = (long)rows * nt;
        k_gemv_generic<<<(unsigned)((warps * 32 + 127) / 128), 128, 0, st>>>(g, fmt, nt);
        return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
    }
    if (nt == 1 && gemv_tma_ok(fmt, g)) {
        TmaGroup grp = {};
        grp.W = g.W; grp.S = g.S; grp.x = x; grp.y = y; grp.rows = rows; grp.sel = -1;
        return gemv_tma(fmt, &grp, 1, cols, g.blk_r, g.blk_c, nullptr, st);
    }
    return gemv_reg(g, fmt, nt, st);
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

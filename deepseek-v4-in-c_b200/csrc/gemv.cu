// gemv.cu - GEMV / skinny GEMM against HBM-resident weights in the
// checkpoint's storage formats: FP8 128x128, FP4 1x32, BF16, F32.
//
// Replaces the reference's k_mmq_fp8 / k_mmq_fp8_n (src/cuda/dsv4_cuda.cu:
// 93-230) and widens it to the four formats dsv4_mmq dispatches on
// (src/core/dsv4_matmul.c:516-591). Three kernels:
//   k_gemv_group  batch 1, up to 16 matrices per launch (mixed formats,
//                 routed experts picked on the device, optional SwiGLU pair
//                 epilogue), one wave of two blocks per SM, each block a tile
//                 of rows of one matrix. Every model matrix (FP8 with
//                 power-of-two blocks of >= 128 columns, FP4 whose scales keep
//                 the f16 decode exact, BF16; <= 64 units per row) runs on the
//                 tensor cores (mma_tile, gemv_mma.cuh: mma.sync m16n8k16 with
//                 x split into three exact pieces, the order written there).
//                 Other shapes take the CUDA-core tile (group_tile): every
//                 half-warp owns one or two 256-byte segments of the row, keeps
//                 their x in registers and walks the tile's rows with eight
//                 16-byte weight loads in flight per thread; segment sums meet
//                 in shared memory and are added in double in segment order
//                 (gemv_core.cuh).
//   k_gemv_nt     nt tokens per weight pass (the batched dsv4_cuda_mmq_n), and
//                 batch-1 shapes whose scale blocks are narrower than a lane;
//                 the segment order of gemv_core.cuh.
//   k_gemv_generic any other shape (rows not a multiple of 16 bytes).
// Each matrix has one order per shape class, independent of the grid, the
// group it runs in and the launch, so a token's result never depends on how
// its GEMVs were batched.
#include <stdlib.h>
#include <string.h>

#include "gemv_core.cuh"
#include "internal.h"

namespace dsv4b {

constexpr int kGemvThreads = 256;           // 16 half-warps per block
constexpr int kGemvSmem = 32 * 1024;        // a block's segment sums
constexpr int kMmaTileSmem = 112 * 1024;    // a tensor-core tile's whole shared memory (two blocks per SM)
constexpr int kMmaTileSmemMT = 220 * 1024;  // a multi-token tile's when its x fragments leave no room for two
constexpr int kGemvMaxTr = 512;

// SwiGLU with the reference's asymmetric clamp (src/core/dsv4_ops.c:60-78):
// up clamped to +-limit, gate from above only; limit <= 0 disables both.
__device__ __forceinline__ float swiglu_pair(float g, float u, float limit)
{
    if (limit > 0.0f) {
        u = fmaxf(fminf(u, limit), -limit);
        g = fminf(g, limit);
    }
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

__device__ __forceinline__ uint8_t ld_nc_u8(const uint8_t *p)
{
    unsigned short v;
    asm volatile("ld.global.nc.u8 %0, [%1];" : "=h"(v) : "l"(p));
    return (uint8_t)v;
}

// The lane's q when its E elements lie in one scale block (one flush).
template <int FMT>
__device__ __forceinline__ float lane_q1(const uint4 &w, const float4 *x, float s)
{
    float sv[8] = {s, s, s, s, s, s, s, s};
    return lane_q<FMT>(w, x, sv, 1u << (Fmt<FMT>::NS - 1));
}

// ------------------------------------------------------------ k_gemv_group

struct TilePtrs {
    const uint8_t *W, *S, *W2, *S2;
};

// Async copy of 16 bytes global -> shared, L1 bypassed; valid == false
// zero-fills the destination and reads nothing.
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool valid)
{
    const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa), "l"(gmem), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Pipeline depth in row steps: NST * SPH 16-byte copies in flight per thread.
template <int SPH>
constexpr int kStages = 8 / SPH;
// Segments per chunk (16 half-warps x SPH): FP4 keeps one segment per
// half-warp, since two segments' x would take 64 registers.
template <int FMT>
constexpr int kChunkSegs = FMT == DSV4B_WFP4 ? 16 : 32;
constexpr int kGemvRing = 8 * kGemvThreads * 16;        // weight ring bytes
constexpr int kGemvSRing = 8 * 16 * 16;                 // FP4 scale ring bytes

// Segments [chunk0, chunk0 + cseg) of every virtual row of one tile. Each
// half-warp owns SPH segments (their x in registers) and walks its rows
// through a ring of kStages<SPH> row steps: every lane copies its own 16
// bytes of each row into the ring and later reads back exactly those bytes,
// so a lane only waits for its own copies. FP4 scales (16 contiguous bytes
// per row and segment) are copied by lane 0 of the half-warp and shared
// after a __syncwarp.
template <int FMT, int SPH>
__device__ __forceinline__ void group_chunk(const GemvItem &it, const TilePtrs &t, int tile, int nvr,
                                            int chunk0, int cseg, int nseg, float *ssum, uint4 *wring,
                                            uint4 *sring, bool sasync)
{
    using F = Fmt<FMT>;
    constexpr int NS = F::NS, E = F::E, NST = kStages<SPH>;
    const int hws = (cseg + SPH - 1) / SPH, rs = 16 / hws;
    const int tid = threadIdx.x, hw = tid >> 4, li = tid & 15;
    const int slot = hw / hws, grp = hw - slot * hws;
    if (slot >= rs) return;
    const unsigned hm = half_mask();
    const int rb = it.rowbytes, trh = it.tr >> 1;
    int seg[SPH], off[SPH], scol[SPH];
    bool lv[SPH], sv[SPH];
    float4 xr[SPH][NS];
#pragma unroll
    for (int j = 0; j < SPH; j++) {
        seg[j] = chunk0 + grp * SPH + j;
        sv[j] = seg[j] < chunk0 + cseg;
        off[j] = seg[j] * 256 + 16 * li;
        lv[j] = sv[j] && off[j] < rb;
        scol[j] = F::SC ? (((off[j] >> 4) * E) >> it.lbc) : 0;
    }
    const int K = slot < nvr ? (nvr - slot + rs - 1) / rs : 0;   // row steps of this slot
    auto locate = [&](int k, int &row, const uint8_t *&Wm, const uint8_t *&Sm) -> bool {
        const int v = slot + k * rs;
        const bool second = it.pair && v >= trh;
        row = it.pair ? tile * trh + (second ? v - trh : v) : tile * it.tr + v;
        Wm = second ? t.W2 : t.W;
        Sm = second ? t.S2 : t.S;
        return v < nvr && row < it.rows;
    };
    auto issue = [&](int k) {
        if (k < K) {
            int row;
            const uint8_t *Wm, *Sm;
            const bool rv = locate(k, row, Wm, Sm);
            const int st = k % NST;
#pragma unroll
            for (int j = 0; j < SPH; j++) {
                const bool ok = rv && lv[j];
                cp_async16(&wring[(st * SPH + j) * kGemvThreads + tid], ok ? Wm + (size_t)row * rb + off[j] : t.W, ok);
                if (FMT == DSV4B_WFP4 && sasync && li == 0) {
                    const bool oks = rv && sv[j];
                    cp_async16(&sring[(st * SPH + j) * 16 + hw], oks ? Sm + (size_t)row * it.sc + scol[j] : t.W, oks);
                }
            }
        }
        cp_commit();
    };
    // the weights do not depend on the previous kernel: start streaming them,
    // then wait for it before reading x
#pragma unroll
    for (int k = 0; k < NST - 1; k++) issue(k);
    pdl_wait();
#pragma unroll
    for (int j = 0; j < SPH; j++) {
        const int e0 = (off[j] >> 4) * E;
#pragma unroll
        for (int k = 0; k < NS; k++)
            xr[j][k] = lv[j] ? ld_f4(it.x + e0 + 4 * k) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int k = 0; k < K; k++) {
        issue(k + NST - 1);
        cp_wait<NST - 1>();
        __syncwarp(hm);
        int row;
        const uint8_t *Wm, *Sm;
        const bool rv = locate(k, row, Wm, Sm);
        const int v = slot + k * rs, st = k % NST;
#pragma unroll
        for (int j = 0; j < SPH; j++) {
            const bool ok = rv && lv[j];
            const uint4 w = wring[(st * SPH + j) * kGemvThreads + tid];
            float s = 1.0f;
            if (F::SC && ok) {
                if (FMT == DSV4B_WFP4 && sasync)
                    s = e8m0(reinterpret_cast<const uint8_t *>(&sring[(st * SPH + j) * 16 + hw])[li]);
                else
                    s = e8m0(__ldg(Sm + (size_t)(row >> it.lbr) * it.sc + scol[j]));
            }
            float q = lane_q1<FMT>(w, xr[j], s);
            q = seg_sum16(q, hm);
            if (li == 0 && rv && sv[j]) ssum[v * (nseg + 1) + seg[j]] = q;
        }
        __syncwarp(hm);
    }
    cp_wait<0>();
}

}  // namespace dsv4b

#include "gemv_mma.cuh"

namespace dsv4b {

template <int FMT>
__device__ __forceinline__ void group_tile(const GemvItem &it, int tile, unsigned char *smem)
{
    TilePtrs t = {it.W, it.S, it.W2, it.S2};
    if (it.wtab) {
        pdl_wait();                  // the selection comes from the previous kernel
        const int e = __ldcg(it.sel + it.slot);
        t.W = it.wtab[e];
        t.S = it.stab ? it.stab[e] : nullptr;
        if (it.pair) {
            t.W2 = it.w2tab[e];
            t.S2 = it.s2tab ? it.s2tab[e] : nullptr;
        }
    }
    const int nseg = (it.rowbytes + 255) >> 8;
    const int nvr = it.tr;
    uint4 *wring = reinterpret_cast<uint4 *>(smem);
    uint4 *sring = reinterpret_cast<uint4 *>(smem + kGemvRing);
    float *ssum = reinterpret_cast<float *>(smem + kGemvRing + kGemvSRing);
    // FP4 scale rows copy 16 bytes per segment when every segment is whole
    const bool sasync = FMT == DSV4B_WFP4 && (it.sc & 15) == 0 && ((uintptr_t)t.S & 15) == 0 &&
                        (!it.pair || ((uintptr_t)t.S2 & 15) == 0);
    constexpr int CMAX = kChunkSegs<FMT>;
    for (int c0 = 0; c0 < nseg; c0 += CMAX) {
        const int cseg = min(CMAX, nseg - c0);
        if constexpr (CMAX > 16) {
            if (cseg > 16) {
                group_chunk<FMT, 2>(it, t, tile, nvr, c0, cseg, nseg, ssum, wring, sring, sasync);
                continue;
            }
        }
        group_chunk<FMT, 1>(it, t, tile, nvr, c0, cseg, nseg, ssum, wring, sring, sasync);
    }
    pdl_wait();                      // idle half-warps too: y is written below
    __syncthreads();
    const int nreal = it.pair ? it.tr >> 1 : it.tr;
    for (int r = threadIdx.x; r < nreal; r += blockDim.x) {
        const int row = tile * nreal + r;
        if (row >= it.rows) break;
        const float *sr = ssum + r * (nseg + 1);
        double tot = 0.0;
        for (int s = 0; s < nseg; s++) tot = __dadd_rn(tot, (double)sr[s]);
        float a = (float)tot;
        if (it.pair) {
            const float *s2 = ssum + (r + nreal) * (nseg + 1);
            double t2 = 0.0;
            for (int s = 0; s < nseg; s++) t2 = __dadd_rn(t2, (double)s2[s]);
            a = swiglu_pair(a, (float)t2, it.limit);
        }
        it.y[row] = a;
    }
}

// NP: token pairs a tensor-core item may carry (0: one token, the batch-1
// launches, with the pair logic compiled out; 1: up to two; 2: up to four).
template <int NP>
__global__ void __launch_bounds__(kGemvThreads, 2)
k_gemv_group(const __grid_constant__ GemvBatch b)
{
    extern __shared__ __align__(16) unsigned char gsm[];
    pdl_trigger();
    int i = 0;
    while (i + 1 < b.n && (int)blockIdx.x >= b.it[i + 1].tile0) i++;
    const GemvItem &it = b.it[i];
    const int tile = (int)blockIdx.x - it.tile0;
    if (it.mma) {
        if (it.fmt == DSV4B_WFP8) mma_tile<DSV4B_WFP8, NP>(it, tile, gsm);
        else if (it.fmt == DSV4B_WFP4) mma_tile<DSV4B_WFP4, NP>(it, tile, gsm);
        else mma_tile<DSV4B_WBF16, NP>(it, tile, gsm);
        return;
    }
    switch (it.fmt) {
    case DSV4B_WF32: group_tile<DSV4B_WF32>(it, tile, gsm); break;
    case DSV4B_WBF16: group_tile<DSV4B_WBF16>(it, tile, gsm); break;
    case DSV4B_WFP8: group_tile<DSV4B_WFP8>(it, tile, gsm); break;
    default: group_tile<DSV4B_WFP4>(it, tile, gsm); break;
    }
}

// --------------------------------------------------------------- k_gemv_nt

struct NtArgs {
    const uint8_t *W, *S;
    const float *x;
    float *y;
    int rows, cols, sc, lbr, lbc, rowbytes;
    long xstride, ystride;
};

// One warp: one row x NT tokens. Half-warp h takes segments h, h+2, ...;
// lane li its 16 bytes of each. Segment sums fold into lane 0's double totals
// in segment order (segment 2m from half 0, then 2m+1 from half 1).
template <int FMT, int NT>
__global__ void __launch_bounds__(128)
k_gemv_nt(NtArgs g)
{
    pdl_trigger();
    pdl_wait();
    using F = Fmt<FMT>;
    constexpr int NS = F::NS, E = F::E;
    const int lane = threadIdx.x & 31, half = lane >> 4, li = lane & 15;
    const int row = (int)((blockIdx.x * (unsigned)blockDim.x + threadIdx.x) >> 5);
    if (row >= g.rows) return;
    const int rb = g.rowbytes, nseg = (rb + 255) >> 8;
    const uint8_t *wr = g.W + (size_t)row * rb;
    double tot[NT];
#pragma unroll
    for (int t = 0; t < NT; t++) tot[t] = 0.0;
    for (int m0 = 0; m0 < nseg; m0 += 4) {
        uint4 w[2];
        bool lv[2];
        int e0[2];
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const int seg = m0 + 2 * j + half, off = seg * 256 + 16 * li;
            lv[j] = seg < nseg && off < rb;
            e0[j] = (off >> 4) * E;
            w[j] = lv[j] ? ld_stream16(wr + off) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int j = 0; j < 2; j++) {
            float s[NS];
            uint32_t fm = 1u << (NS - 1);
            if (F::SC) {
                fm = flush_mask<FMT>(e0[j], g.lbc);
#pragma unroll
                for (int k = 0; k < NS; k++)
                    s[k] = lv[j] ? e8m0(ld_nc_u8(g.S + (size_t)(row >> g.lbr) * g.sc + ((e0[j] + 4 * k) >> g.lbc)))
                                 : 1.0f;
            } else {
#pragma unroll
                for (int k = 0; k < NS; k++) s[k] = 1.0f;
            }
            float q[NT];
#pragma unroll
            for (int t = 0; t < NT; t++) {
                float4 xv[NS];
#pragma unroll
                for (int k = 0; k < NS; k++)
                    xv[k] = lv[j] ? ld_f4(g.x + (size_t)t * g.xstride + e0[j] + 4 * k)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
                q[t] = lv[j] ? lane_q<FMT>(w[j], xv, s, fm) : 0.0f;
            }
            const int sev = m0 + 2 * j;
#pragma unroll
            for (int t = 0; t < NT; t++) {
                const float v = seg_sum16(q[t], 0xffffffffu);
                const float vodd = __shfl_sync(0xffffffffu, v, 16);
                if (lane == 0) {
                    if (sev < nseg) tot[t] = __dadd_rn(tot[t], (double)v);
                    if (sev + 1 < nseg) tot[t] = __dadd_rn(tot[t], (double)vodd);
                }
            }
        }
    }
    if (lane == 0)
#pragma unroll
        for (int t = 0; t < NT; t++) g.y[(size_t)t * g.ystride + row] = (float)tot[t];
}

// ----------------------------------------------------------- k_gemv_generic

// Any shape: one warp per (row, token), scalar loads, exact products summed in
// double. Only reached by shapes whose rows are not 16-byte multiples (the
// reference's hand-sized test matrices); every model matrix takes the others.
__global__ void k_gemv_generic(NtArgs g, int fmt, int blk_r, int blk_c, int nt)
{
    pdl_trigger();
    pdl_wait();
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
        if (fmt >= DSV4B_WFP8) s = (double)e8m0(g.S[(o / blk_r) * g.sc + c / blk_c]);
        acc = __fma_rn((double)w * s, (double)x[c], acc);
    }
    acc = warp_sum_d(acc);
    if (lane == 0) g.y[(size_t)t * g.ystride + o] = (float)acc;
}

// --------------------------------------------------------------------- host

static int lane_elems(int fmt)
{
    return fmt == DSV4B_WF32 ? 4 : fmt == DSV4B_WBF16 ? 8 : fmt == DSV4B_WFP8 ? 16 : 32;
}

static int log2_exact(int v)
{
    if (v <= 0 || (v & (v - 1))) return -1;
    int l = 0;
    while ((1 << l) < v) l++;
    return l;
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

bool gemv_vectorizable(int fmt, const void *W, int cols, int blk_r, int blk_c, const float *x, long xstride)
{
    const size_t rb = row_bytes(fmt, cols);
    if (rb % 16 || ((uintptr_t)W & 15) || ((uintptr_t)x & 15) || (xstride & 3)) return false;
    // scale blocks: powers of two, and a sub-step's 4 elements inside one block
    if (fmt >= DSV4B_WFP8 && (log2_exact(blk_c) < 2 || log2_exact(blk_r) < 0)) return false;
    return true;
}

bool gemv_item(GemvItem &it, int fmt, const void *W, const uint8_t *S, int rows, int cols, int blk_r,
               int blk_c, const float *x, float *y, bool f16s)
{
    memset(&it, 0, sizeof it);
    blk_r = blk_r > 0 ? blk_r : 1;
    blk_c = blk_c > 0 ? blk_c : 1;
    if (!gemv_vectorizable(fmt, W, cols, blk_r, blk_c, x, 0)) return false;
    if (fmt >= DSV4B_WFP8 && blk_c < lane_elems(fmt)) return false;   // a lane's elements share one scale
    it.W = (const uint8_t *)W;
    it.S = S;
    it.x = x;
    it.y = y;
    it.fmt = fmt;
    it.rows = rows;
    it.cols = cols;
    it.rowbytes = (int)row_bytes(fmt, cols);
    it.sc = fmt >= DSV4B_WFP8 ? (cols + blk_c - 1) / blk_c : 0;
    it.lbr = fmt >= DSV4B_WFP8 ? log2_exact(blk_r) : 0;
    it.lbc = fmt >= DSV4B_WFP8 ? log2_exact(blk_c) : 30;
    it.mma = gemv_mma_shape(fmt, cols, blk_r, blk_c, f16s) ? 1 : 0;
    return true;
}

bool gemv_mma_shape(int fmt, int cols, int blk_r, int blk_c, bool f16s)
{
    if (fmt == DSV4B_WF32) return false;
    const int uc = mma_unit_cols(fmt);
    if (cols % uc || cols / uc > kMmaMaxBlocks) return false;
    if (fmt == DSV4B_WFP8) return blk_c >= 128 && log2_exact(blk_c) >= 0 && log2_exact(blk_r) >= 0;
    if (fmt == DSV4B_WFP4) return f16s && blk_c == 32 && blk_r == 1;
    return true;
}

int gemv_item_tokens(GemvItem &it, int want, long xts, long yts)
{
    if (!it.mma || want <= 1) return 1;
    const int nb = it.cols / mma_unit_cols(it.fmt), minrows = it.pair ? 32 : 16;
    int k = want < 4 ? want : 4;
    while (k > 1 && mma_smem(it.fmt, nb, minrows, k) > (size_t)kMmaTileSmemMT) k--;
    if (k > 1) {
        it.nt = k;
        it.xts = (int)xts;
        it.yts = (int)yts;
    }
    return k;
}

bool fp4_scales_f16(const uint8_t *s, size_t n)
{
    for (size_t i = 0; i < n; i++)
        if (s[i] < 127 - 23 || s[i] > 127 + 1) return false;
    return true;
}

int gemv_group(GemvItem *items, int n, cudaStream_t st)
{
    if (n <= 0) return 0;
    if (n > kGemvMaxItems) return -1;
    static int nsm = 0;
    if (!nsm) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
        if (nsm <= 0) nsm = 148;
    }
    double total = 0.0;
    for (int i = 0; i < n; i++) total += (double)items[i].rows * items[i].rowbytes * (items[i].pair ? 2 : 1);
    // one wave of two resident blocks per SM, each streaming 16-256 KB: a
    // block's prologue (x fragments, pipeline fill) is paid once for as much
    // streaming as it can get, and no second wave leaves SMs idle at the end
    double target = total / (2.0 * nsm);
    target = target < 16384.0 ? 16384.0 : (target > 262144.0 ? 262144.0 : target);
    GemvBatch b;
    b.n = n;
    int blocks = 0;
    size_t smem = 0;
    for (int i = 0; i < n; i++) {
        GemvItem &it = items[i];
        it.tile0 = blocks;
        if (it.rows <= 0) {
            it.tr = 2;
            b.it[i] = it;
            continue;
        }
        if (it.mma) {
            const int nb = it.cols / mma_unit_cols(it.fmt), ntk = it.nt > 1 ? it.nt : 1;
            // a multi-token item keeps two resident blocks per SM where its
            // smallest tile fits them (measured: 8 % off a batch-32 step), else
            // takes one block's whole budget
            const bool two = ntk == 1 || mma_smem(it.fmt, nb, it.pair ? 32 : 16, ntk) <= (size_t)kMmaTileSmem;
            const int budget = two ? kMmaTileSmem : kMmaTileSmemMT;
            // a multiple of 16 virtual rows, within the shared memory budget
            int cap = (int)((budget - mma_smem(it.fmt, nb, 0, ntk)) / (64 * ntk)) & ~15;
            cap = cap < 512 ? cap : 512;
            if (cap < 16) return -1;
            int tr = ((int)(target / it.rowbytes) + 15) & ~15;
            tr = tr < 16 ? 16 : (tr > cap ? cap : tr);
            if (it.pair) {
                tr = (tr + 31) & ~31;
                if (tr > cap) tr = cap & ~31;
                if (tr < 32) tr = 32;
                if (tr / 2 > it.rows) tr = ((2 * it.rows + 31) & ~31);
            } else if (tr > it.rows) {
                tr = (it.rows + 15) & ~15;
            }
            it.tr = tr;
            const int per = it.pair ? tr / 2 : tr;
            blocks += (it.rows + per - 1) / per;
            const size_t sm = mma_smem(it.fmt, nb, tr, ntk);
            if (sm > smem) smem = sm;
            b.it[i] = it;
            continue;
        }
        const int nseg = (it.rowbytes + 255) >> 8;
        const int cmax = it.fmt == DSV4B_WFP4 ? 16 : 32;
        const int cseg = nseg < cmax ? nseg : cmax, sph = cseg > 16 ? 2 : 1;
        const int hws = (cseg + sph - 1) / sph, gran = (16 / hws) * (8 / sph);   // virtual rows per pass
        int cap = (int)(kGemvSmem / ((size_t)(nseg + 1) * 4));
        cap = cap < kGemvMaxTr ? cap : kGemvMaxTr;
        if (cap < 2) return -1;
        int tr = (int)(target / it.rowbytes);
        tr = tr < 1 ? 1 : tr;
        tr = (tr + gran - 1) / gran * gran;
        tr = tr < cap ? tr : cap;
        if (it.pair) {
            tr &= ~1;
            if (tr < 2) tr = 2;
            if (tr / 2 > it.rows) tr = 2 * it.rows;
        } else if (tr > it.rows) {
            tr = it.rows;
        }
        it.tr = tr;
        const int per = it.pair ? tr / 2 : tr;      // real rows per block
        blocks += (it.rows + per - 1) / per;
        const size_t sm = kGemvRing + kGemvSRing + (size_t)tr * (nseg + 1) * 4;
        if (sm > smem) smem = sm;
        b.it[i] = it;
    }
    if (!blocks) return 0;
    int maxnt = 1;
    for (int i = 0; i < n; i++) maxnt = items[i].nt > maxnt ? items[i].nt : maxnt;
    auto kern = maxnt > 2 ? k_gemv_group<2> : maxnt > 1 ? k_gemv_group<1> : k_gemv_group<0>;
    if (smem_optin(kern, maxnt > 1 ? kMmaTileSmemMT : kMmaTileSmem)) return -1;
    return launch(kern, dim3(blocks), dim3(kGemvThreads), smem, st, b) ==
                   cudaSuccess
               ? 0
               : -1;
}

template <int FMT, int NT>
static void launch_nt(const NtArgs &a, cudaStream_t st)
{
    const int blocks = (a.rows + 3) / 4;
    launch(k_gemv_nt<FMT, NT>, dim3(blocks), dim3(128), 0, st, a);
}

template <int FMT>
static void launch_fmt(const NtArgs &a, int nt, cudaStream_t st)
{
    switch (nt) {
    case 1: launch_nt<FMT, 1>(a, st); break;
    case 2: launch_nt<FMT, 2>(a, st); break;
    case 3: launch_nt<FMT, 3>(a, st); break;
    case 4: launch_nt<FMT, 4>(a, st); break;
    case 5: launch_nt<FMT, 5>(a, st); break;
    case 6: launch_nt<FMT, 6>(a, st); break;
    case 7: launch_nt<FMT, 7>(a, st); break;
    default: launch_nt<FMT, 8>(a, st); break;
    }
}

int gemv(int fmt, float *y, long ystride, const float *x, long xstride, const void *W, const uint8_t *S,
         int rows, int cols, int blk_r, int blk_c, int nt, cudaStream_t st, bool f16s)
{
    if (rows <= 0 || cols <= 0 || nt <= 0) return 0;
    if (fmt == DSV4B_WFP4 && (cols & 1)) return -1;
    blk_r = blk_r > 0 ? blk_r : 1;
    blk_c = blk_c > 0 ? blk_c : 1;
    NtArgs a = {};
    a.W = (const uint8_t *)W;
    a.S = S;
    a.x = x;
    a.y = y;
    a.rows = rows;
    a.cols = cols;
    a.rowbytes = (int)row_bytes(fmt, cols);
    a.sc = fmt >= DSV4B_WFP8 ? (cols + blk_c - 1) / blk_c : 0;
    a.lbr = fmt >= DSV4B_WFP8 ? log2_exact(blk_r) : 0;
    a.lbc = fmt >= DSV4B_WFP8 ? log2_exact(blk_c) : 30;
    a.xstride = xstride;
    a.ystride = ystride;
    if (!gemv_vectorizable(fmt, W, cols, blk_r, blk_c, x, xstride)) {
        const long warps = (long)rows * nt;
        launch(k_gemv_generic, dim3((unsigned)((warps * 32 + 127) / 128)), dim3(128), 0, st, a, fmt, blk_r, blk_c, nt);
        return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
    }
    if (nt == 1 && ystride >= rows) {
        GemvItem it;
        if (gemv_item(it, fmt, W, S, rows, cols, blk_r, blk_c, x, y, f16s)) return gemv_group(&it, 1, st);
    }
    if (gemv_mma_shape(fmt, cols, blk_r, blk_c, f16s)) {
        // the tensor-core order: every token as its own item (same kernel and
        // arithmetic as a batch-1 call), up to 16 per launch
        for (int t0 = 0; t0 < nt; t0 += kGemvMaxItems) {
            const int k = (nt - t0 < kGemvMaxItems) ? nt - t0 : kGemvMaxItems;
            GemvItem it[kGemvMaxItems];
            for (int t = 0; t < k; t++)
                if (!gemv_item(it[t], fmt, W, S, rows, cols, blk_r, blk_c, x + (size_t)(t0 + t) * xstride,
                               y + (size_t)(t0 + t) * ystride, f16s))
                    return -1;
            if (gemv_group(it, k, st)) return -1;
        }
        return 0;
    }
    for (int t0 = 0; t0 < nt; t0 += 8) {
        const int k = (nt - t0 < 8) ? nt - t0 : 8;
        NtArgs b = a;
        b.x = x + (size_t)t0 * xstride;
        b.y = y + (size_t)t0 * ystride;
        switch (fmt) {
        case DSV4B_WF32: launch_fmt<DSV4B_WF32>(b, k, st); break;
        case DSV4B_WBF16: launch_fmt<DSV4B_WBF16>(b, k, st); break;
        case DSV4B_WFP8: launch_fmt<DSV4B_WFP8>(b, k, st); break;
        default: launch_fmt<DSV4B_WFP4>(b, k, st); break;
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

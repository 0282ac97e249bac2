// gemv_tma.cu - batch-1 GEMV as a TMA bulk-copy weight stream.
//
// The decode step is a weight stream: every matrix is read once per token and
// each byte feeds one or two multiply-adds. This kernel keeps HBM busy with
// few threads: one producer lane issues cp.async.bulk copies (non-multicast,
// local HBM only) of 16 rows x 1 KB weight chunks, plus the matching x chunk
// and, for FP4, the chunk's scale bytes, into a 7-stage shared-memory ring
// guarded by mbarriers; eight consumer warps decode and multiply out of shared
// memory, each lane reusing its x unit across 4 rows.
//
// Work is the flat list of (16-row tile, 1 KB chunk) items of one or more
// matrices, cut into one contiguous range per CTA (one CTA per SM), so skinny
// matrices split their K dimension across SMs instead of leaving most SMs
// idle. A tile whose chunks span CTAs parks its segment sums in a per-device
// scratch slot and the last CTA to arrive (an atomic counter) folds it; the
// fold order is the canonical one of gemv_core.cuh either way, so the result
// does not depend on the split.
//
// Every wait is bounded (about one second of %globaltimer); on expiry the
// kernel records an error code in the workspace and drains without blocking.
#include "gemv_core.cuh"
#include "internal.h"

namespace dsv4b {

constexpr int TR = 16;          // rows per tile
constexpr int KC = 1024;        // weight bytes per row per stage
constexpr int NSTAGE = 7;
constexpr int NCW = 8;          // consumer warps
constexpr int NSEGMAX = 128;    // 256-byte segments per row: rows <= 32 KB
constexpr int W_BYTES = TR * KC;
constexpr int X_BYTES = KC * 32 / 4;       // x of one chunk at 2 elements/byte
constexpr int S_BYTES = TR * KC / 16;      // FP4 scales of one chunk
constexpr int STAGE_BYTES = W_BYTES + X_BYTES + S_BYTES;
constexpr int SEG_BYTES = 2 * TR * NSEGMAX * 4;
constexpr int SMEM_BYTES = NSTAGE * STAGE_BYTES + SEG_BYTES + 2 * NSTAGE * 8;

struct TmaArgs {
    TmaGroup grp[kTmaMaxGroups];
    int tile0[kTmaMaxGroups + 1];
    int ngroups, rowbytes, blk_r, blk_c, sc, nchunks, nseg;
    long nitems;
    const int *sel;
    float *segbuf;
    int *cnt;
    int *err;
};

__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *b, int count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t *b, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n}"
                 : "=r"(ok)
                 : "r"(smem_u32(b)), "r"(parity)
                 : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t gtimer()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait on an mbarrier phase. Gives up after ~1 s (or at once when
// another thread of the CTA already gave up), recording `code`.
__device__ __noinline__ bool mbar_wait(uint64_t *b, uint32_t parity, int *err, int code,
                                       volatile int *abort_flag)
{
    if (mbar_try(b, parity)) return true;
    const uint64_t t0 = gtimer();
    for (uint32_t it = 0; it < 0x7fffffffu; it++) {
        if (mbar_try(b, parity)) return true;
        if ((it & 63) == 0) {
            if (*abort_flag) return false;
            if (gtimer() - t0 > 1000000000ull) {
                atomicOr(err, code);
                *abort_flag = 1;
                return false;
            }
        }
    }
    return false;
}
__device__ __forceinline__ void tma_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void consumer_sync()
{
    asm volatile("bar.sync 1, %0;" ::"r"(NCW * 32) : "memory");
}

// The CTA whose item range contains `item` (ranges are [b*N/G, (b+1)*N/G)).
__device__ __forceinline__ int block_of(long item, long N, int G)
{
    long b = (item * G) / N;
    while (b + 1 < G && ((b + 1) * N) / G <= item) b++;
    while (b > 0 && (b * N) / G > item) b--;
    return (int)b;
}

struct ItemInfo {
    int T, c, gi, row0, nrows, cb;
};

__device__ __forceinline__ ItemInfo item_info(const TmaArgs &a, long it)
{
    ItemInfo f;
    f.T = (int)(it / a.nchunks);
    f.c = (int)(it % a.nchunks);
    int gi = 0;
    while (gi + 1 < a.ngroups && f.T >= a.tile0[gi + 1]) gi++;
    f.gi = gi;
    f.row0 = (f.T - a.tile0[gi]) * TR;
    f.nrows = min(TR, a.grp[gi].rows - f.row0);
    f.cb = min(KC, a.rowbytes - f.c * KC);
    return f;
}

template <int FMT>
__global__ void __launch_bounds__((NCW + 1) * 32, 1)
k_gemv_tma(const __grid_constant__ TmaArgs a)
{
    constexpr int EPU = Fmt<FMT>::EPU;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *stages = smem;
    float *segs = reinterpret_cast<float *>(smem + NSTAGE * STAGE_BYTES);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + NSTAGE * STAGE_BYTES + SEG_BYTES);
    uint64_t *empty = full + NSTAGE;
    __shared__ int s_last;
    __shared__ volatile int s_abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long N = a.nitems;
    const int G = gridDim.x;
    const long lo = (long)blockIdx.x * N / G, hi = (long)(blockIdx.x + 1) * N / G;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NSTAGE; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == NCW) {
        // ------------------------------------------------------ producer
        if (lane == 0) {
            for (long it = lo; it < hi; it++) {
                const long i = it - lo;
                const int s = (int)(i % NSTAGE);
                const uint32_t ph = (uint32_t)((i / NSTAGE) & 1);
                if (i >= NSTAGE && !mbar_wait(&empty[s], ph ^ 1u, a.err, 1, &s_abort)) break;
                const ItemInfo f = item_info(a, it);
                const TmaGroup &gr = a.grp[f.gi];
                const uint8_t *W = gr.W, *S = gr.S;
                if (gr.sel >= 0) {
                    const long e = a.sel[gr.sel];
                    W += e * gr.wstride;
                    if (S) S += e * gr.sstride;
                }
                const uint32_t xb = (uint32_t)(f.cb * EPU / 4);
                const uint32_t sb = (FMT == DSV4B_WFP4) ? (uint32_t)(f.cb / 16) : 0u;
                uint8_t *st = stages + (size_t)s * STAGE_BYTES;
                mbar_expect_tx(&full[s], (uint32_t)f.nrows * ((uint32_t)f.cb + sb) + xb);
                for (int r = 0; r < f.nrows; r++)
                    tma_load(st + r * KC, W + (size_t)(f.row0 + r) * a.rowbytes + (size_t)f.c * KC,
                             (uint32_t)f.cb, &full[s]);
                tma_load(st + W_BYTES, gr.x + (size_t)f.c * (KC / 16) * EPU, xb, &full[s]);
                if (FMT == DSV4B_WFP4)
                    for (int r = 0; r < f.nrows; r++)
                        tma_load(st + W_BYTES + X_BYTES + r * (KC / 16),
                                 S + (size_t)(f.row0 + r) * a.sc + (size_t)f.c * (KC / 16), sb, &full[s]);
            }
        }
        return;
    }

    // --------------------------------------------------------- consumers
    const int half = lane >> 4, li = lane & 15;
    const int task = warp * 2 + half, rg = task >> 2, sg = task & 3;
    const int ctid = threadIdx.x;
    bool dead = false;
    int buf = 0;
    for (long it = lo; it < hi; it++) {
        const long i = it - lo;
        const int s = (int)(i % NSTAGE);
        const uint32_t ph = (uint32_t)((i / NSTAGE) & 1);
        const ItemInfo f = item_info(a, it);
        // Every lane acquires the phase itself; the verdict is made uniform so
        // the shuffles below never run with part of the warp missing.
        bool ok = dead ? false : mbar_wait(&full[s], ph, a.err, 2, &s_abort);
        if (!__all_sync(0xffffffffu, ok)) dead = true;
        float *sg_buf = segs + buf * TR * NSEGMAX;
        if (!dead) {
            const uint8_t *st = stages + (size_t)s * STAGE_BYTES;
            const float *xs = reinterpret_cast<const float *>(st + W_BYTES);
            const int off = sg * 256 + li * 16;
            const bool uok = off < f.cb;
            const uint8_t *S = a.grp[f.gi].S;
            if (FMT == DSV4B_WFP8 && a.grp[f.gi].sel >= 0) S += (long)a.sel[a.grp[f.gi].sel] * a.grp[f.gi].sstride;
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const int lr = rg * 4 + r;
                const bool ok = uok && lr < f.nrows;
                float q = 0.0f;
                if (ok) {
                    const uint4 w = *reinterpret_cast<const uint4 *>(st + lr * KC + off);
                    q = unit_dot<FMT>(w, xs + (off >> 4) * EPU);
                    if constexpr (FMT == DSV4B_WFP8) {
                        const int col = f.c * KC + off;
                        q = __fmul_rn(q, e8m0(__ldg(S + ((f.row0 + lr) / a.blk_r) * a.sc + col / a.blk_c)));
                    } else if constexpr (FMT == DSV4B_WFP4) {
                        q = __fmul_rn(q, e8m0(st[W_BYTES + X_BYTES + lr * (KC / 16) + (off >> 4)]));
                    }
                }
                const float v = seg_sum16(q);
                if (li == 0 && sg * 256 < f.cb && lr < f.nrows) sg_buf[lr * NSEGMAX + f.c * 4 + sg] = v;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);

        if (f.c == a.nchunks - 1 || it == hi - 1) {
            // ----------------------------------------------- tile end
            consumer_sync();
            const long t_first = (long)f.T * a.nchunks;
            const int c_lo = (t_first >= lo) ? 0 : (int)(lo - t_first);
            const int c_hi = f.c + 1;
            float *y = a.grp[f.gi].y + f.row0;
            if (c_lo == 0 && c_hi == a.nchunks) {
                if (ctid < f.nrows && !dead) {
                    double tot = 0.0;
                    for (int j = 0; j < a.nseg; j++) tot = __dadd_rn(tot, (double)sg_buf[ctid * NSEGMAX + j]);
                    y[ctid] = (float)tot;
                }
            } else {
                const int slot = block_of(t_first, N, G);
                float *sb = a.segbuf + (size_t)slot * TR * NSEGMAX;
                const int jlo = c_lo * 4, jhi = min(c_hi * 4, a.nseg), nj = jhi - jlo;
                for (int k = ctid; k < f.nrows * nj; k += NCW * 32) {
                    const int r = k / nj, j = jlo + k % nj;
                    sb[r * NSEGMAX + j] = sg_buf[r * NSEGMAX + j];
                }
                __threadfence();
                consumer_sync();
                if (ctid == 0) {
                    const int prev = atomicAdd(a.cnt + slot, c_hi - c_lo);
                    s_last = (prev + (c_hi - c_lo) == a.nchunks);
                }
                consumer_sync();
                if (s_last) {
                    __threadfence();
                    if (ctid < f.nrows && !dead) {
                        double tot = 0.0;
                        for (int j = 0; j < a.nseg; j++)
                            tot = __dadd_rn(tot, (double)__ldcg(sb + ctid * NSEGMAX + j));
                        y[ctid] = (float)tot;
                    }
                    if (ctid == 0) a.cnt[slot] = 0;
                }
            }
            buf ^= 1;
        }
    }
}

static Workspace g_ws = {};
Workspace &workspace() { return g_ws; }

int workspace_init()
{
    if (g_ws.segbuf) return 0;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_ws.nsm, cudaDevAttrMultiProcessorCount, dev);
    g_ws.slots = g_ws.nsm;
    if (cudaMalloc(&g_ws.segbuf, (size_t)g_ws.slots * TR * NSEGMAX * sizeof(float)) != cudaSuccess) return -1;
    if (cudaMalloc(&g_ws.cnt, (size_t)(g_ws.slots + 1) * sizeof(int)) != cudaSuccess) return -1;
    g_ws.err = g_ws.cnt + g_ws.slots;
    if (cudaMemset(g_ws.cnt, 0, (size_t)(g_ws.slots + 1) * sizeof(int)) != cudaSuccess) return -1;
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : -1;
}

void workspace_free()
{
    if (g_ws.segbuf) cudaFree(g_ws.segbuf);
    if (g_ws.cnt) cudaFree(g_ws.cnt);
    g_ws = Workspace{};
}

bool gemv_tma_ok(int fmt, const GemvArgs &g)
{
    if (!g_ws.segbuf) return false;
    if (g.rowbytes % 16 || g.rowbytes > NSEGMAX * 256) return false;
    if (((uintptr_t)g.W & 15) || ((uintptr_t)g.x & 15)) return false;
    if (fmt == DSV4B_WFP4 && (g.rowbytes % 256 || g.sc % 16 || ((uintptr_t)g.S & 15))) return false;
    return true;
}

template <int FMT>
static int launch_tma(const TmaArgs &a, cudaStream_t st)
{
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(k_gemv_tma<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
            cudaSuccess)
            return -1;
        attr = true;
    }
    const int grid = (int)((a.nitems < g_ws.nsm) ? a.nitems : g_ws.nsm);
    k_gemv_tma<FMT><<<grid, (NCW + 1) * 32, SMEM_BYTES, st>>>(a);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

int gemv_tma(int fmt, const TmaGroup *grp, int ngroups, int cols, int blk_r, int blk_c,
             const int *sel_idx, cudaStream_t st)
{
    if (ngroups < 1 || ngroups > kTmaMaxGroups || !g_ws.segbuf) return -1;
    TmaArgs a = {};
    a.ngroups = ngroups;
    a.rowbytes = (int)row_bytes(fmt, cols);
    a.blk_r = blk_r > 0 ? blk_r : 1;
    a.blk_c = blk_c > 0 ? blk_c : 1;
    a.sc = fmt >= DSV4B_WFP8 ? (cols + a.blk_c - 1) / a.blk_c : 0;
    a.nchunks = (a.rowbytes + KC - 1) / KC;
    a.nseg = (a.rowbytes + 255) / 256;
    int tiles = 0;
    for (int g = 0; g < ngroups; g++) {
        a.grp[g] = grp[g];
        a.tile0[g] = tiles;
        tiles += (grp[g].rows + TR - 1) / TR;
    }
    a.tile0[ngroups] = tiles;
    a.nitems = (long)tiles * a.nchunks;
    if (a.nitems == 0) return 0;
    a.sel = sel_idx;
    a.segbuf = g_ws.segbuf;
    a.cnt = g_ws.cnt;
    a.err = g_ws.err;
    switch (fmt) {
    case DSV4B_WF32: return launch_tma<DSV4B_WF32>(a, st);
    case DSV4B_WBF16: return launch_tma<DSV4B_WBF16>(a, st);
    case DSV4B_WFP8: return launch_tma<DSV4B_WFP8>(a, st);
    default: return launch_tma<DSV4B_WFP4>(a, st);
    }
}

}  // namespace dsv4b

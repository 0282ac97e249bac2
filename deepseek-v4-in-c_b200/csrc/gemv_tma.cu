// gemv_tma.cu - batch-1 GEMV as a TMA bulk-copy weight stream.
//
// The decode step is a weight stream: every matrix is read once per token and
// each byte feeds one or two multiply-adds. Rows of a matrix are contiguous,
// so R consecutive whole rows (up to 32 KB) are ONE contiguous block, and one
// cp.async.bulk copy (non-multicast, local HBM only) moves a whole stage.
// Measured on this part, bulk copies of >= 4 KB stream a 29 MB matrix at the
// same rate as a full-occupancy load kernel, while 1 KB copies lose ~25%.
//
// One CTA per SM: a producer lane loads every x the launch needs into shared
// memory once, then streams stages of R rows through a 4-deep ring guarded by
// mbarriers. Eight consumer warps (16 half-warps) split each stage into
// (row pair, segment phase) tasks, so each lane's x registers serve two rows.
// Per-(row, segment) sums land in shared memory; after a consumer barrier the
// stage's rows are folded in segment order (gemv_core.cuh) by R threads while
// the other warps move on. Work is the flat list of R-row items of up to 16
// matrices (a grouped launch: e.g. the w1/w3 of six routed experts), cut into
// one contiguous range per CTA.
//
// Every wait is bounded (about one second of %globaltimer); on expiry the
// kernel records an error code in the workspace and drains without blocking.
#include "gemv_core.cuh"
#include "internal.h"

namespace dsv4b {

constexpr int NSTAGE = 4;
constexpr int NCW = 8;                    // consumer warps
constexpr int STAGE_MAX = 32768;          // weight bytes per stage
constexpr int SCALE_MAX = 2048;           // FP4 scale bytes per stage
constexpr int X_MAX = 65536;              // bytes of x held in shared memory
constexpr int SEGS_MAX = STAGE_MAX / 256 + 32; // (row, segment) sums per stage
constexpr int SMEM_BYTES = NSTAGE * (STAGE_MAX + SCALE_MAX) + X_MAX + 2 * SEGS_MAX * 4 + (2 * NSTAGE + 1) * 8;

struct TmaArgs {
    TmaGroup grp[kTmaMaxGroups];
    int item0[kTmaMaxGroups + 1];   // first item of each group
    int xoff[kTmaMaxGroups];        // float offset of each group's x in shared memory
    int nx;                         // distinct x vectors to load
    int xsrc[kTmaMaxGroups];        // group whose x fills slot i
    int xslot_off[kTmaMaxGroups];
    int ngroups, rowbytes, cols, R, nseg, lbr, lbc, sc, nitems;
    const int *sel;
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

// Walks a CTA's items (R-row groups) in order.
struct ItemIter {
    int it, gi, row0, nrows;
    __device__ __forceinline__ void start(const TmaArgs &a, int i)
    {
        it = i;
        gi = 0;
        while (gi + 1 < a.ngroups && it >= a.item0[gi + 1]) gi++;
        fill(a);
    }
    __device__ __forceinline__ void next(const TmaArgs &a)
    {
        ++it;
        while (gi + 1 < a.ngroups && it >= a.item0[gi + 1]) gi++;
        fill(a);
    }
    __device__ __forceinline__ void fill(const TmaArgs &a)
    {
        row0 = (it - a.item0[gi]) * a.R;
        nrows = min(a.R, a.grp[gi].rows - row0);
    }
};

template <int FMT>
__global__ void __launch_bounds__((NCW + 1) * 32, 1)
k_gemv_tma(const __grid_constant__ TmaArgs a)
{
    using F = Fmt<FMT>;
    constexpr int NS = F::NSTEP, SB = F::SB;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *wst = smem;                                               // NSTAGE x STAGE_MAX
    uint8_t *sst = smem + NSTAGE * STAGE_MAX;                          // NSTAGE x SCALE_MAX
    float *xsm = reinterpret_cast<float *>(sst + NSTAGE * SCALE_MAX);  // X_MAX
    float *segs = xsm + X_MAX / 4;                                     // 2 x SEGS_MAX
    uint64_t *full = reinterpret_cast<uint64_t *>(segs + 2 * SEGS_MAX);
    uint64_t *empty = full + NSTAGE;
    uint64_t *xbar = empty + NSTAGE;
    __shared__ volatile int s_abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int N = a.nitems, G = gridDim.x;
    const int lo = (int)(((long long)blockIdx.x * N) / G), hi = (int)(((long long)(blockIdx.x + 1) * N) / G);
    if (threadIdx.x == 0) {
        for (int s = 0; s < NSTAGE; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        mbar_init(xbar, 1);
        s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const int xbytes = a.cols * 4;

    if (warp == NCW) {
        // ------------------------------------------------------ producer
        if (lane == 0) {
            mbar_expect_tx(xbar, (uint32_t)(xbytes * a.nx));
            for (int i = 0; i < a.nx; i++)
                tma_load(xsm + a.xslot_off[i], a.grp[a.xsrc[i]].x, (uint32_t)xbytes, xbar);
            ItemIter f;
            f.start(a, lo);
            for (int it = lo; it < hi; it++, f.next(a)) {
                const int i = it - lo, s = i % NSTAGE;
                const uint32_t ph = (uint32_t)((i / NSTAGE) & 1);
                if (i >= NSTAGE && !mbar_wait(&empty[s], ph ^ 1u, a.err, 1, &s_abort)) break;
                const TmaGroup &gr = a.grp[f.gi];
                const uint8_t *W = gr.W, *S = gr.S;
                if (gr.sel >= 0) {
                    const long e = a.sel[gr.sel];
                    W += e * gr.wstride;
                    if (S) S += e * gr.sstride;
                }
                const uint32_t wb = (uint32_t)(f.nrows * a.rowbytes);
                const uint32_t sb = (FMT == DSV4B_WFP4) ? (uint32_t)(f.nrows * a.sc) : 0u;
                mbar_expect_tx(&full[s], wb + sb);
                tma_load(wst + (size_t)s * STAGE_MAX, W + (size_t)f.row0 * a.rowbytes, wb, &full[s]);
                if (FMT == DSV4B_WFP4)
                    tma_load(sst + (size_t)s * SCALE_MAX, S + (size_t)f.row0 * a.sc, sb, &full[s]);
            }
        }
        return;
    }

    // --------------------------------------------------------- consumers
    const int half = lane >> 4, li = lane & 15, hw = warp * 2 + half;   // half-warp 0..15
    const int npair = a.R >> 1, nphase = 16 / npair;
    const int pair = hw % npair, phase = hw / npair;
    bool dead = false;
    bool ok = mbar_wait(xbar, 0, a.err, 4, &s_abort);
    if (!__all_sync(0xffffffffu, ok)) dead = true;
    ItemIter f;
    f.start(a, lo);
    for (int it = lo; it < hi; it++, f.next(a)) {
        const int i = it - lo, s = i % NSTAGE;
        const uint32_t ph = (uint32_t)((i / NSTAGE) & 1);
        // Every lane acquires the phase itself; the verdict is made uniform so
        // the shuffles below never run with part of the warp missing.
        ok = dead ? false : mbar_wait(&full[s], ph, a.err, 2, &s_abort);
        if (!__all_sync(0xffffffffu, ok)) dead = true;
        float *sg = segs + (i & 1) * SEGS_MAX;
        if (!dead) {
            const uint8_t *wsm = wst + (size_t)s * STAGE_MAX;
            const uint8_t *ssm = sst + (size_t)s * SCALE_MAX;
            const float *xg = xsm + a.xoff[f.gi];
            const int r0 = pair * 2;
            const uint8_t *S8 = nullptr;
            if constexpr (FMT == DSV4B_WFP8) {
                const TmaGroup &gr = a.grp[f.gi];
                S8 = gr.S;
                if (gr.sel >= 0) S8 += (long)a.sel[gr.sel] * gr.sstride;
            }
            for (int j = phase; j < a.nseg; j += nphase) {
                const int seg0 = j * 256;
                int nvalid = 0;
#pragma unroll
                for (int k = 0; k < NS; k++) nvalid += (seg0 + SB * (16 * k + li) < a.rowbytes) ? 1 : 0;
                const int e0 = seg0 * 4 / SB;
                const StepMasks m = step_masks<FMT>(e0, li, nvalid, a.lbc);
                float4 xv[NS];
#pragma unroll
                for (int k = 0; k < NS; k++)
                    xv[k] = (k < nvalid) ? *reinterpret_cast<const float4 *>(xg + e0 + 4 * (16 * k + li))
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int r = 0; r < 2; r++) {
                    const int lr = r0 + r;
                    float q = 0.0f;
                    if (lr < f.nrows) {
                        uint4 w[NS];
                        float sc[NS];
#pragma unroll
                        for (int k = 0; k < NS; k++) {
                            const int off = seg0 + SB * (16 * k + li);
                            w[k] = (k < nvalid) ? load_step<FMT>(wsm + lr * a.rowbytes + off) : make_uint4(0u, 0u, 0u, 0u);
                            sc[k] = 1.0f;
                            if constexpr (FMT == DSV4B_WFP8)
                                if (k < nvalid)
                                    sc[k] = e8m0(__ldg(S8 + ((f.row0 + lr) >> a.lbr) * a.sc + ((e0 + 4 * (16 * k + li)) >> a.lbc)));
                            if constexpr (FMT == DSV4B_WFP4)
                                if (k < nvalid) sc[k] = e8m0(ssm[lr * a.sc + ((e0 + 4 * (16 * k + li)) >> a.lbc)]);
                        }
                        q = lane_q<FMT>(w, xv, sc, m);
                    }
                    const float v = seg_sum16(q);
                    if (li == 0 && lr < f.nrows) sg[lr * a.nseg + j] = v;
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        consumer_sync();
        // fold this stage's rows: row r by lane (r >> 3) of warp (r & 7)
        const int fr = (lane < 2) ? (warp + 8 * lane) : a.R;
        if (!dead && fr < f.nrows) {
            double tot = 0.0;
            for (int j = 0; j < a.nseg; j++) tot = __dadd_rn(tot, (double)sg[fr * a.nseg + j]);
            a.grp[f.gi].y[f.row0 + fr] = (float)tot;
        }
    }
}

static Workspace g_ws = {};
Workspace &workspace() { return g_ws; }

int workspace_init()
{
    if (g_ws.cnt) return 0;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_ws.nsm, cudaDevAttrMultiProcessorCount, dev);
    g_ws.slots = g_ws.nsm;
    if (cudaMalloc(&g_ws.cnt, (size_t)(g_ws.slots + 1) * sizeof(int)) != cudaSuccess) return -1;
    g_ws.err = g_ws.cnt + g_ws.slots;
    g_ws.segbuf = nullptr;
    if (cudaMemset(g_ws.cnt, 0, (size_t)(g_ws.slots + 1) * sizeof(int)) != cudaSuccess) return -1;
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : -1;
}

void workspace_free()
{
    if (g_ws.cnt) cudaFree(g_ws.cnt);
    g_ws = Workspace{};
}

// Rows per stage: as many whole rows as fit 32 KB, at least 2 (x reuse) and
// at most 16 (one row pair per half-warp).
static int rows_per_stage(int rowbytes)
{
    int R = 16;
    while (R > 2 && R * rowbytes > STAGE_MAX) R >>= 1;
    return (R * rowbytes <= STAGE_MAX) ? R : 0;
}

bool gemv_tma_ok(int fmt, const GemvArgs &g)
{
    if (!g_ws.cnt) return false;
    if (g.rowbytes % 16 || rows_per_stage(g.rowbytes) == 0) return false;
    if ((size_t)g.cols * 4 > (size_t)X_MAX || (g.cols * 4) % 16) return false;
    if (((uintptr_t)g.W & 15) || ((uintptr_t)g.x & 15)) return false;
    if (fmt == DSV4B_WFP4) {
        const int R = rows_per_stage(g.rowbytes);
        if ((R * g.sc) % 16 || R * g.sc > SCALE_MAX || ((uintptr_t)g.S & 15) || g.sc % 16) return false;
    }
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
    const int grid = (a.nitems < g_ws.nsm) ? a.nitems : g_ws.nsm;
    k_gemv_tma<FMT><<<grid, (NCW + 1) * 32, SMEM_BYTES, st>>>(a);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

int gemv_tma(int fmt, const TmaGroup *grp, int ngroups, int cols, int blk_r, int blk_c,
             const int *sel_idx, cudaStream_t st)
{
    if (ngroups < 1 || ngroups > kTmaMaxGroups || !g_ws.cnt) return -1;
    TmaArgs a = {};
    a.ngroups = ngroups;
    a.cols = cols;
    a.rowbytes = (int)row_bytes(fmt, cols);
    a.R = rows_per_stage(a.rowbytes);
    if (a.R == 0) return -1;
    a.nseg = (a.rowbytes + 255) / 256;
    const int br = blk_r > 0 ? blk_r : 1, bc = blk_c > 0 ? blk_c : 1;
    a.lbr = 0;
    while ((1 << a.lbr) < br) a.lbr++;
    a.lbc = 0;
    while ((1 << a.lbc) < bc) a.lbc++;
    if (fmt < DSV4B_WFP8) a.lbc = 30;
    a.sc = fmt >= DSV4B_WFP8 ? (cols + bc - 1) / bc : 0;
    int items = 0;
    for (int g = 0; g < ngroups; g++) {
        a.grp[g] = grp[g];
        a.item0[g] = items;
        items += (grp[g].rows + a.R - 1) / a.R;
        // one shared-memory slot per distinct x
        int slot = -1;
        for (int i = 0; i < a.nx; i++)
            if (a.grp[a.xsrc[i]].x == grp[g].x) slot = i;
        if (slot < 0) {
            slot = a.nx++;
            a.xsrc[slot] = g;
            a.xslot_off[slot] = slot * cols;
        }
        a.xoff[g] = a.xslot_off[slot];
    }
    if ((size_t)a.nx * cols * 4 > (size_t)X_MAX) return -1;
    a.item0[ngroups] = items;
    a.nitems = items;
    if (items == 0) return 0;
    a.sel = sel_idx;
    a.err = g_ws.err;
    switch (fmt) {
    case DSV4B_WF32: return launch_tma<DSV4B_WF32>(a, st);
    case DSV4B_WBF16: return launch_tma<DSV4B_WBF16>(a, st);
    case DSV4B_WFP8: return launch_tma<DSV4B_WFP8>(a, st);
    default: return launch_tma<DSV4B_WFP4>(a, st);
    }
}

}  // namespace dsv4b

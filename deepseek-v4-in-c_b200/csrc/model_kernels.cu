// model_kernels.cu - the support ops of one decode token on the device.
//
// Every position-dependent quantity (the RoPE row, the KV ring slot, the
// compressor phase, how many compressed rows exist, the window list) is read
// from a device StepState rather than passed by the host, so a whole token is
// a fixed sequence of launches that one CUDA graph can replay for every
// position. Each kernel restates its reference function (cited) with the same
// operation order; reductions over a vector are block-wide in double where the
// reference sums in double.
#include <limits.h>

#include "common.cuh"
#include "model.h"

namespace dsv4b {

__device__ __forceinline__ double block_sum_d(double v, double *red)
{
    v = warp_sum_d(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    double t = 0.0;
    if (threadIdx.x == 0) {
        for (int i = 0; i < nw; i++) t += red[i];
        red[32] = t;
    }
    __syncthreads();
    return red[32];
}

// block_sum_d over the first nw warps only, synchronised by named barrier
// bar (the other warps of the block are busy elsewhere).
__device__ __forceinline__ double part_sum_d(double v, double *red, int nw, int bar)
{
    v = warp_sum_d(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nw * 32) : "memory");
    if (lane == 0) red[w] = v;
    asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nw * 32) : "memory");
    double t = 0.0;
    if (threadIdx.x == 0) {
        for (int i = 0; i < nw; i++) t += red[i];
        red[32] = t;
    }
    asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nw * 32) : "memory");
    return red[32];
}

// dsv4_embed_row (include/dsv4/dsv4.h:300-314), replicated hc times
// (src/cli/dsv4_run.c:449-450). Sequence blockIdx.y of a batch: its step
// state st[y], its residual at h + y hc hidden.
__global__ void k_embed(float *h, const void *table, int wdt, const StepState *st, int hidden, int hc)
{
    pdl_trigger();
    pdl_wait();
    h += (size_t)blockIdx.y * hc * hidden;
    const long tok = st[blockIdx.y].token;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += gridDim.x * blockDim.x) {
        float v;
        if (wdt == DSV4B_WBF16)
            v = __uint_as_float((uint32_t)reinterpret_cast<const uint16_t *>(table)[tok * hidden + i] << 16);
        else
            v = reinterpret_cast<const float *>(table)[tok * hidden + i];
        for (int j = 0; j < hc; j++) h[(size_t)j * hidden + i] = v;
    }
}

// mixes[m] = (float)(fn[m] . x) * rs, rs = (float)(1/sqrt(mean(x^2) + eps)),
// both sums in double over the flattened hc*hidden vector
// (src/core/dsv4_hc.c:118-129, src/cli/dsv4_run.c:97-107). grid = rows.
__global__ void k_hc_mix(float *mixes, const float *fn, const float *x, int n, float eps)
{
    pdl_trigger();
    pdl_wait();
    __shared__ double red[33];
    const float *row = fn + (size_t)blockIdx.x * n;
    double sq = 0.0, dot = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const double xv = (double)x[i];
        sq = __fma_rn(xv, xv, sq);
        dot = __fma_rn((double)row[i], xv, dot);
    }
    sq = block_sum_d(sq, red);
    dot = block_sum_d(dot, red);
    if (threadIdx.x == 0) {
        const float rs = (float)(1.0 / sqrt(sq / (double)n + (double)eps));
        mixes[blockIdx.x] = __fmul_rn((float)dot, rs);
    }
}

__device__ __forceinline__ float sigm(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }

// dsv4_hc_split_sinkhorn (src/core/dsv4_hc.c:50-102) then y = sum_j pre[j] x[j]
// in double (:135-140). One block.
__global__ void k_hc_finish(float *y, float *post, float *comb, const float *mixes, const float *x,
                            const float *scale, const float *base, int hc, int hidden, int iters, float eps)
{
    pdl_trigger();
    pdl_wait();
    __shared__ float pre[DSV4B_MAX_HC], cb[DSV4B_MAX_HC * DSV4B_MAX_HC];
    if (threadIdx.x == 0) {
        for (int j = 0; j < hc; j++) pre[j] = __fadd_rn(sigm(__fadd_rn(__fmul_rn(mixes[j], scale[0]), base[j])), eps);
        for (int j = 0; j < hc; j++)
            post[j] = __fmul_rn(2.0f, sigm(__fadd_rn(__fmul_rn(mixes[j + hc], scale[1]), base[j + hc])));
        for (int j = 0; j < hc; j++)
            for (int k = 0; k < hc; k++) {
                const int o = j * hc + k + hc * 2;
                cb[j * hc + k] = __fadd_rn(__fmul_rn(mixes[o], scale[2]), base[o]);
            }
        for (int j = 0; j < hc; j++) {
            float *r = cb + j * hc;
            float mx = r[0];
            for (int k = 1; k < hc; k++) if (r[k] > mx) mx = r[k];
            double sum = 0.0;
            for (int k = 0; k < hc; k++) { r[k] = expf(r[k] - mx); sum += (double)r[k]; }
            const float inv = (float)(1.0 / sum);
            for (int k = 0; k < hc; k++) r[k] = __fadd_rn(__fmul_rn(r[k], inv), eps);
        }
        const int npass = iters > 1 ? iters : 1;
        for (int pass = 0; pass < npass; pass++) {
            if (pass > 0)
                for (int j = 0; j < hc; j++) {
                    double rs = 0.0;
                    for (int k = 0; k < hc; k++) rs += (double)cb[j * hc + k];
                    const float d = __fadd_rn((float)rs, eps);
                    for (int k = 0; k < hc; k++) cb[j * hc + k] = __fdiv_rn(cb[j * hc + k], d);
                }
            for (int k = 0; k < hc; k++) {
                double cs = 0.0;
                for (int j = 0; j < hc; j++) cs += (double)cb[j * hc + k];
                const float d = __fadd_rn((float)cs, eps);
                for (int j = 0; j < hc; j++) cb[j * hc + k] = __fdiv_rn(cb[j * hc + k], d);
            }
        }
        for (int i = 0; i < hc * hc; i++) comb[i] = cb[i];
    }
    __syncthreads();
    for (int d = blockIdx.x * blockDim.x + threadIdx.x; d < hidden; d += gridDim.x * blockDim.x) {
        double acc = 0.0;
        for (int j = 0; j < hc; j++) acc = __dadd_rn(acc, __dmul_rn((double)pre[j], (double)x[(size_t)j * hidden + d]));
        y[d] = (float)acc;
    }
}

// The Sinkhorn split of the comb mixes (src/core/dsv4_hc.c:63-101) on one
// warp: lane l holds comb[l / hc][l % hc]; a row's (column's) entries are
// fetched by shuffles and summed in double in index order, rounded to float,
// plus eps, as the reference does, and every entry divided (float, correctly
// rounded). HC > 0 fixes hc at compile time, so the shuffles of a sum are
// issued together; HC = 0 takes hc at run time. hc * hc <= 32.
template <int HC>
__device__ __forceinline__ void sinkhorn_warp(float *comb, const float *mixes, float scale2, const float *base,
                                              int hc_rt, int iters, float eps)
{
    const int hc = HC > 0 ? HC : hc_rt;
    const int l = threadIdx.x & 31, j = l / hc, k = l % hc;
    const bool act = l < hc * hc;
    const unsigned full = 0xffffffffu;
    const int o = 2 * hc + (act ? l : 0);
    float v = __fadd_rn(__fmul_rn(mixes[o], scale2), base[o]);
    const int rj = act ? j * hc : 0, ck = act ? k : 0;
    constexpr int NU = HC > 0 ? HC : 8;           // unroll bound
    auto row_sum = [&](float x) {
        float g[NU];
#pragma unroll
        for (int kk = 0; kk < NU; kk++) g[kk] = kk < hc ? __shfl_sync(full, x, rj + kk) : 0.0f;
        double s = 0.0;
#pragma unroll
        for (int kk = 0; kk < NU; kk++)
            if (kk < hc) s = __dadd_rn(s, (double)g[kk]);
        return s;
    };
    auto col_sum = [&](float x) {
        float g[NU];
#pragma unroll
        for (int jj = 0; jj < NU; jj++) g[jj] = jj < hc ? __shfl_sync(full, x, jj * hc + ck) : 0.0f;
        double s = 0.0;
#pragma unroll
        for (int jj = 0; jj < NU; jj++)
            if (jj < hc) s = __dadd_rn(s, (double)g[jj]);
        return s;
    };
    // first pass: row softmax (max, exp, double sum), + eps, then columns
    float mx;
    {
        float g[NU];
#pragma unroll
        for (int kk = 0; kk < NU; kk++) g[kk] = kk < hc ? __shfl_sync(full, v, rj + kk) : -INFINITY;
        mx = g[0];
#pragma unroll
        for (int kk = 1; kk < NU; kk++)
            if (kk < hc) mx = fmaxf(mx, g[kk]);
    }
    const float e = expf(v - mx);
    v = __fadd_rn(__fmul_rn(e, (float)(1.0 / row_sum(e))), eps);
    v = __fdiv_rn(v, __fadd_rn((float)col_sum(v), eps));
    // the remaining iters - 1 passes: rows, then columns
    for (int pass = 1; pass < iters; pass++) {
        v = __fdiv_rn(v, __fadd_rn((float)row_sum(v), eps));
        v = __fdiv_rn(v, __fadd_rn((float)col_sum(v), eps));
    }
    if (act) comb[l] = v;
}

// The whole mHC pre-mix of one sub-layer in one launch, with the sub-layer's
// RMSNorm folded in (src/core/dsv4_hc.c:118-140 with dsv4_hc_split_sinkhorn
// :50-102, then src/core/dsv4_ops.c:25-32 when norm_w is given), optionally
// preceded by the previous sub-layer's post-mix (k_hc_post, and before it the
// MoE combine k_combine), each thread finishing the one residual element it
// then mixes:
//   every block: [post step: blk[d] (or sum_k wts[k] acc[k][d] + accs[d] in
//                float, as k_combine), xout[i] = post_in[j] blk[d] +
//                sum_l comb_in[l][j] x[l][d] in double, as k_hc_post]; per
//                column the products fn[m][i] * x[i] and x[i]^2 (float),
//                summed per block in a fixed order (32 columns in float, then
//                8 such sums in double), written to part[block][0..nmix];
//   last block:  the partials summed in block order (double), mixes, the
//                pre weights; then, at the same time, warps 0..7 compute
//                y = sum_j pre[j] x[j] and its RMSNorm while warp 8 (layers)
//                computes the post weights and the Sinkhorn split (each lane
//                one comb entry, every row / column fetched by shuffles and
//                summed in double in index order, as the reference does).
// Head mode (post null, nmix = hc) is the head's reduction
// (src/cli/dsv4_run.c:94-116): the sigmoid pre weights only.
// The reference sums these in double; here only the short sums across warps
// and blocks are, which keeps the result within ~1e-7 of it while avoiding
// long chains of double operations. The last block is the one whose arrival
// at *count completes the grid; it resets *count, so the kernel is
// replayable. post_in / comb_in may be the post / comb outputs: every block
// has read them before it arrives at *count. hc * hc <= 32.
// MODE 0: the whole step in one launch (the last block to finish its
// partials runs the tail); MODE 1: the partials only (a batch's first
// launch, no counter, blocks exit); MODE 2: the tail only, block = sequence
// (a batch's second launch). The arithmetic is the same in every mode.
template <bool BATCH, int MODE>
__device__ __forceinline__ void hc_pre_body(const HcPreArgs &a)
{
    constexpr int MIXMAX = kHcPreMixMax, NV = MIXMAX + 1;
    // sequence blockIdx.y (tail: blockIdx.x) of a batch: its own rows of
    // every activation (pointers computed here; the argument block itself is
    // never modified; one sequence: every offset is the constant 0)
    const size_t sq_ = MODE == 2 ? blockIdx.x : (BATCH ? blockIdx.y : 0), wide_ = (size_t)a.hc * a.hidden;
    const int nparts = (int)(wide_ >> 8);           // blocks of the partials (256 columns each)
    float *const yq = a.y + sq_ * a.hidden;
    float *const postq = a.post ? a.post + sq_ * DSV4B_MAX_HC : nullptr;
    float *const combq = a.comb ? a.comb + sq_ * DSV4B_MAX_HC * DSV4B_MAX_HC : nullptr;
    const float *const xq = a.x + sq_ * wide_;
    float *const xoutq = a.xout ? a.xout + sq_ * wide_ : nullptr;
    const float *const blkq = a.blk ? a.blk + sq_ * a.hidden : nullptr;
    const float *const accq = a.acc ? a.acc + sq_ * a.s_ms : nullptr;
    const float *const wtsq = a.wts ? a.wts + sq_ * a.s_ms : nullptr;
    const float *const accsq = a.accs ? a.accs + sq_ * a.s_ms : nullptr;
    const float *const pinq = a.post_in ? a.post_in + sq_ * DSV4B_MAX_HC : nullptr;
    const float *const cinq = a.comb_in ? a.comb_in + sq_ * DSV4B_MAX_HC * DSV4B_MAX_HC : nullptr;
    double *const partq = a.part + sq_ * nparts * NV;
    unsigned *const cntq = a.count + sq_;
    __shared__ float prod[NV][256];
    __shared__ double red8[NV][8];
    __shared__ double tot[NV];
    __shared__ float mixes[MIXMAX], pre[DSV4B_MAX_HC], sbase[MIXMAX], sscale[3];
    __shared__ bool last;
    const int hc = a.hc, hidden = a.hidden, n = hc * hidden, mix = a.nmix, tid = threadIdx.x;
    const bool stepped = blkq || accq;
    pdl_trigger();
    if (tid < mix) sbase[tid] = __ldg(a.base + tid);     // weights: before the wait
    if (tid < (postq ? 3 : 1)) sscale[tid] = __ldg(a.scale + tid);
    // one column per thread of warps 0..7 (the launcher sizes the grid to
    // n / 256; warp 8 only runs the split); its fn column is a weight,
    // fetched before waiting for x
    const bool col = tid < 256;
    const int i = blockIdx.x * 256 + tid;
    const int h4 = hidden >> 2;
    float4 wn[kHcPreYPT];                                // the norm weights of this thread's columns
#pragma unroll
    for (int u = 0; u < kHcPreYPT; u++) {
        const int d4 = tid + u * 256;
        wn[u] = (a.norm_w && col && d4 < h4) ? __ldg(reinterpret_cast<const float4 *>(a.norm_w) + d4)
                                      : make_float4(1.f, 1.f, 1.f, 1.f);
    }
    if constexpr (MODE != 2) {
    float fv[MIXMAX];
#pragma unroll
    for (int m = 0; m < MIXMAX; m++) fv[m] = (m < mix && col && i < n) ? __ldg(a.fn + (size_t)m * n + i) : 0.0f;
    pdl_wait();
    float xv = 0.0f;
    if (col && i < n) {
        if (stepped) {
            const int j = i / hidden, d = i - j * hidden;
            // every load of the step issued before any is used (fixed-size,
            // predicated batches), then the sums in their order
            float b;
            float xl[DSV4B_MAX_HC], cl[DSV4B_MAX_HC];
#pragma unroll
            for (int l = 0; l < DSV4B_MAX_HC; l++) {
                xl[l] = l < hc ? ld_act(xq + (size_t)l * hidden + d) : 0.0f;
                cl[l] = l < hc ? ld_act(cinq + l * hc + j) : 0.0f;
            }
            const float pj = ld_act(pinq + j);
            if (accq) {
                float wv[kMoeMaxTopk], av[kMoeMaxTopk];
#pragma unroll
                for (int k = 0; k < kMoeMaxTopk; k++) {
                    wv[k] = k < a.topk ? ld_act(wtsq + k) : 0.0f;
                    av[k] = k < a.topk ? ld_act(accq + (size_t)k * hidden + d) : 0.0f;
                }
                const float sv = accsq ? ld_act(accsq + d) : 0.0f;
                float o = 0.0f;
#pragma unroll
                for (int k = 0; k < kMoeMaxTopk; k++)
                    if (k < a.topk) o = __fadd_rn(o, __fmul_rn(wv[k], av[k]));
                if (accsq) o = __fadd_rn(o, sv);
                b = o;
            } else {
                b = ld_act(blkq + d);
            }
            double s = __dmul_rn((double)pj, (double)b);
#pragma unroll
            for (int l = 0; l < DSV4B_MAX_HC; l++)
                if (l < hc) s = __dadd_rn(s, __dmul_rn((double)cl[l], (double)xl[l]));
            xv = (float)s;
            xoutq[i] = xv;
        } else {
            xv = ld_act(xq + i);
        }
    }
    if (col) {
#pragma unroll
        for (int m = 0; m < MIXMAX; m++) prod[m][tid] = __fmul_rn(fv[m], xv);
        prod[MIXMAX][tid] = __fmul_rn(xv, xv);
    }
    __syncthreads();
    if (tid < NV * 8) {
        const int m = tid >> 3, w = tid & 7;
        float sacc = 0.0f;
#pragma unroll 8
        for (int k = 0; k < 32; k++) sacc = __fadd_rn(sacc, prod[m][w * 32 + k]);
        red8[m][w] = (double)sacc;
    }
    __syncthreads();
    if (tid < NV) {
        double t = 0.0;
#pragma unroll
        for (int w = 0; w < 8; w++) t += red8[tid][w];
        partq[(size_t)blockIdx.x * NV + tid] = t;
    }
    if constexpr (MODE == 1) return;
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(cntq, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    } else {
        pdl_wait();                                 // the partials of the previous launch
    }
    const float *x = stepped ? xoutq : xq;
    // every block's partials: 8 threads per value each add gridDim/8 blocks,
    // then the 8 sums in order
    const int nblk = nparts, per = (nblk + 7) >> 3;
    if (tid < NV * 8) {
        const int m = tid >> 3, w = tid & 7;
        constexpr int PB = kHcPreBlocks / 8;       // per <= PB: all loads first
        double pv[PB];
#pragma unroll
        for (int k = 0; k < PB; k++) {
            const int bb = w * per + k;
            pv[k] = (k < per && bb < nblk) ? __ldcg(partq + (size_t)bb * NV + m) : 0.0;
        }
        double t = 0.0;
#pragma unroll
        for (int k = 0; k < PB; k++)
            if (k < per && w * per + k < nblk) t += pv[k];
        red8[m][w] = t;
    }
    __syncthreads();
    if (tid < NV) {
        double t = 0.0;
#pragma unroll
        for (int w = 0; w < 8; w++) t += red8[tid][w];
        tot[tid] = t;
    }
    __syncthreads();
    if (MODE == 0 && tid == 0) *cntq = 0u;
    if (tid < 32) {
        const float rs = __fdiv_rn(1.0f, __fsqrt_rn((float)(tot[MIXMAX] / (double)n) + a.rms_eps));
        if (tid < mix) mixes[tid] = __fmul_rn((float)tot[tid], rs);
        __syncwarp();
        if (tid < hc) pre[tid] = __fadd_rn(sigm(__fadd_rn(__fmul_rn(mixes[tid], sscale[0]), sbase[tid])), a.hc_eps);
    }
    __syncthreads();
    if (tid >= 256) {
        // the extra warp: post weights and the Sinkhorn split, concurrently
        // with y below (only the next sub-layer's post-mix reads them)
        if (!postq) return;
        const int l = tid - 256;
        if (l < hc) postq[l] = __fmul_rn(2.0f, sigm(__fadd_rn(__fmul_rn(mixes[l + hc], sscale[1]), sbase[l + hc])));
        if (hc == 4)
            sinkhorn_warp<4>(combq, mixes, sscale[2], sbase, 4, a.iters, a.hc_eps);
        else
            sinkhorn_warp<0>(combq, mixes, sscale[2], sbase, hc, a.iters, a.hc_eps);
        return;
    }
    // warps 0..7: y = sum_j pre[j] x[j], four columns per float4, in two
    // batches of loads; then RMSNorm from the registers
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    float4 yv[kHcPreYPT];
    float sq = 0.0f;
    constexpr int YB = kHcPreYPT / 2;
#pragma unroll
    for (int half = 0; half < 2; half++) {
        float4 xw[YB][4];
#pragma unroll
        for (int uu = 0; uu < YB; uu++) {
            const int d4 = tid + (half * YB + uu) * 256;
#pragma unroll
            for (int j = 0; j < 4; j++)
                xw[uu][j] = (d4 < h4 && j < hc) ? __ldcg(x4 + (size_t)j * h4 + d4) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int uu = 0; uu < YB; uu++) {
            const int u = half * YB + uu, d4 = tid + u * 256;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            if (d4 < h4) {
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    if (j < hc) {
                        const float pj = pre[j];
                        acc.x = __fmaf_rn(pj, xw[uu][j].x, acc.x);
                        acc.y = __fmaf_rn(pj, xw[uu][j].y, acc.y);
                        acc.z = __fmaf_rn(pj, xw[uu][j].z, acc.z);
                        acc.w = __fmaf_rn(pj, xw[uu][j].w, acc.w);
                    }
                }
                sq = __fmaf_rn(acc.x, acc.x, sq);
                sq = __fmaf_rn(acc.y, acc.y, sq);
                sq = __fmaf_rn(acc.z, acc.z, sq);
                sq = __fmaf_rn(acc.w, acc.w, sq);
            }
            yv[u] = acc;
        }
    }
    float inv = 1.0f;
    if (a.norm_w) {
        __shared__ double nred[33];
        const double ssq = part_sum_d((double)sq, nred, 8, 1);
        inv = __fdiv_rn(1.0f, __fsqrt_rn((float)(ssq / (double)hidden) + a.rms_eps));
    }
    float4 *y4 = reinterpret_cast<float4 *>(yq);
#pragma unroll
    for (int u = 0; u < kHcPreYPT; u++) {
        const int d4 = tid + u * 256;
        if (d4 < h4) {
            float4 o = yv[u];
            if (a.norm_w) {
                const float4 wv = wn[u];
                o = make_float4(__fmul_rn(wv.x, __fmul_rn(o.x, inv)), __fmul_rn(wv.y, __fmul_rn(o.y, inv)),
                                __fmul_rn(wv.z, __fmul_rn(o.z, inv)), __fmul_rn(wv.w, __fmul_rn(o.w, inv)));
            }
            y4[d4] = o;
        }
    }
}

__global__ void __launch_bounds__(288) k_hc_pre(const __grid_constant__ HcPreArgs a) { hc_pre_body<false, 0>(a); }
__global__ void __launch_bounds__(288) k_hc_pre_batch(const __grid_constant__ HcPreArgs a) { hc_pre_body<true, 0>(a); }
__global__ void __launch_bounds__(288) k_hc_part_batch(const __grid_constant__ HcPreArgs a) { hc_pre_body<true, 1>(a); }
__global__ void __launch_bounds__(288) k_hc_tail_batch(const __grid_constant__ HcPreArgs a) { hc_pre_body<true, 2>(a); }

// The head's reduction: a sigmoid gate per copy, one scalar scale, no
// Sinkhorn (src/cli/dsv4_run.c:94-116). One block.
__global__ void k_hc_head_finish(float *y, const float *mixes, const float *x, const float *scale,
                                 const float *base, int hc, int hidden, float eps)
{
    pdl_trigger();
    pdl_wait();
    __shared__ float pre[DSV4B_MAX_HC];
    if (threadIdx.x < hc) {
        const int j = threadIdx.x;
        pre[j] = __fadd_rn(sigm(__fadd_rn(__fmul_rn(mixes[j], scale[0]), base[j])), eps);
    }
    __syncthreads();
    for (int d = threadIdx.x; d < hidden; d += blockDim.x) {
        double acc = 0.0;
        for (int j = 0; j < hc; j++) acc = __dadd_rn(acc, __dmul_rn((double)pre[j], (double)x[(size_t)j * hidden + d]));
        y[d] = (float)acc;
    }
}

// y[k][d] = post[k] x[d] + sum_j comb[j][k] res[j][d], in double
// (src/core/dsv4_hc.c:149-162).
__global__ void k_hc_post(float *y, const float *x, const float *res, const float *post, const float *comb,
                          int hc, int hidden)
{
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= hc * hidden) return;
    const int k = i / hidden, d = i % hidden;
    double acc = __dmul_rn((double)post[k], (double)x[d]);
    for (int j = 0; j < hc; j++)
        acc = __dadd_rn(acc, __dmul_rn((double)comb[j * hc + k], (double)res[(size_t)j * hidden + d]));
    y[i] = (float)acc;
}

// RMSNorm (src/core/dsv4_ops.c:25-32): double sum of squares, eps on the mean,
// y = w * (x * inv). One block per vector (block b: the n values at b n);
// y may alias x.
__global__ void k_rmsnorm(float *y, const float *x, const float *w, int n, float eps)
{
    pdl_trigger();
    pdl_wait();
    y += (size_t)blockIdx.x * n;
    x += (size_t)blockIdx.x * n;
    __shared__ double red[33];
    double s = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s = __fma_rn((double)x[i], (double)x[i], s);
    s = block_sum_d(s, red);
    const float inv = (float)(1.0 / sqrt(s / (double)n + (double)eps));
    for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = __fmul_rn(w[i], __fmul_rn(x[i], inv));
}

// One head: optional unweighted RMS (the q path,
// src/model/dsv4_layer.c:224-231), then RoPE at pos. The whole block.
__device__ void head_norm_rope(float *h, int width, int rd, const float *cs, const float *sn, int pos, int inverse,
                               int do_norm, float eps, double *red)
{
    if (do_norm) {
        double s = 0.0;
        for (int i = threadIdx.x; i < width; i += blockDim.x) s = __fma_rn((double)h[i], (double)h[i], s);
        s = block_sum_d(s, red);
        const float inv = (float)(1.0 / sqrt(s / (double)width + (double)eps));
        for (int i = threadIdx.x; i < width; i += blockDim.x) h[i] = __fmul_rn(h[i], inv);
        __syncthreads();
    }
    rope_tail(h, width, rd, cs, sn, pos, inverse);
}

// The new KV row: weighted RMSNorm, RoPE at pos, into its window slot
// (src/model/dsv4_layer.c:233-238). The whole block.
// dst: the cache row the finished KV row goes to (its window ring slot, or
// a prefill pass's staging row).
__device__ void kv_finish(float *kv, const float *w, int hd, int rd, const float *cs, const float *sn, int pos,
                          float eps, float *dst, double *red)
{
    double s = 0.0;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) s = __fma_rn((double)kv[i], (double)kv[i], s);
    s = block_sum_d(s, red);
    const float inv = (float)(1.0 / sqrt(s / (double)hd + (double)eps));
    for (int i = threadIdx.x; i < hd; i += blockDim.x) kv[i] = __fmul_rn(w[i], __fmul_rn(kv[i], inv));
    __syncthreads();
    rope_tail(kv, hd, rd, cs, sn, pos, 0);
    __syncthreads();
    for (int i = threadIdx.x; i < hd; i += blockDim.x) dst[i] = kv[i];
}

// cbuf[c], c < hd: column c of an emitted compressed row, the softmax over
// its ns slots in slot order (src/core/dsv4_compress.c), slot s's (value,
// score) from get(s, c); a -inf score is an empty slot, and an all-empty
// column is 0.
template <class Get>
__device__ __forceinline__ void comp_pool(float *cbuf, int hd, int ns, Get get)
{
    for (int c = threadIdx.x; c < hd; c += blockDim.x) {
        float mx = -INFINITY;
        for (int s = 0; s < ns; s++) {
            const float v = get(s, c).y;
            if (v > mx) mx = v;
        }
        float out = 0.0f;
        if (mx != -INFINITY) {
            double den = 0.0, acc = 0.0;
            for (int s = 0; s < ns; s++) {
                const float2 g = get(s, c);
                if (g.y == -INFINITY) continue;
                const double e = (double)expf(g.y - mx);
                den = __dadd_rn(den, e);
                acc = __dadd_rn(acc, __dmul_rn(e, (double)g.x));
            }
            out = (float)(acc / den);
        }
        cbuf[c] = out;
    }
}

// The pooled row's RMSNorm (weights norm) and RoPE at the window's first
// position pos0, written to cache row `row`.
__device__ void comp_finish(float *cache, float *cbuf, const float *norm, int hd, int rd, const float *cs,
                            const float *sn, int pos0, float eps, int row, double *red)
{
    double s = 0.0;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) s = __fma_rn((double)cbuf[i], (double)cbuf[i], s);
    s = block_sum_d(s, red);
    const float inv = (float)(1.0 / sqrt(s / (double)hd + (double)eps));
    for (int i = threadIdx.x; i < hd; i += blockDim.x) cbuf[i] = __fmul_rn(norm[i], __fmul_rn(cbuf[i], inv));
    __syncthreads();
    rope_tail(cbuf, hd, rd, cs, sn, pos0, 0);
    __syncthreads();
    float *dst = cache + (size_t)row * hd;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) dst[i] = cbuf[i];
}

__device__ void compress_step(float *cache, float *kv_state, float *score_state, const float *kv_in,
                              const float *sc_in, const float *ape, const float *norm, int ratio, int hd, int rd,
                              const float *cs, const float *sn, int pos, float eps, int win, int index_topk,
                              int *dyn, float *cbuf, double *red)
{
    // a batch's sequences stand at the same position: sequence 0 writes the
    // shared counts
    if (blockIdx.y != 0) dyn = nullptr;
    const int overlap = (ratio == 4), coff = 1 + overlap, width = coff * hd;
    const int phase = pos % ratio, slot = overlap ? ratio + phase : phase;
    const float *apr = ape + (size_t)phase * width;
    for (int c = threadIdx.x; c < width; c += blockDim.x) {
        kv_state[(size_t)slot * width + c] = kv_in[c];
        score_state[(size_t)slot * width + c] = __fadd_rn(sc_in[c], apr[c]);
    }
    const int avail = (pos + 1) / ratio;
    if (threadIdx.x == 0 && dyn) {
        dyn[0] = avail;
        dyn[1] = avail < index_topk ? avail : index_topk;
    }
    __syncthreads();
    if ((pos + 1) % ratio != 0) return;
    // slot s of the pool: overlap mode takes the previous window's first
    // half-width and the current window's second half-width
    comp_pool(cbuf, hd, overlap ? 2 * ratio : ratio, [&](int s, int c) {
        const size_t off = overlap ? ((s < ratio) ? (size_t)s * width + c : (size_t)s * width + hd + c)
                                   : (size_t)s * width + c;
        return make_float2(kv_state[off], score_state[off]);
    });
    __syncthreads();
    if (overlap) {       // slide: the current window becomes the previous one
        for (int i = threadIdx.x; i < ratio * width; i += blockDim.x) {
            kv_state[i] = kv_state[(size_t)ratio * width + i];
            score_state[i] = score_state[(size_t)ratio * width + i];
        }
    }
    comp_finish(cache, cbuf, norm, hd, rd, cs, sn, pos + 1 - ratio, eps, win + avail - 1, red);
}

// A prefill pass's compressor, token y of the pass (position pos, the pass
// from position p0): its counts {avail, take} at dyn, and, when its position
// closes a window, the compressed row of that window. The row's slots are
// read where the per-token steps would have put them: positions inside the
// pass from the pass's projection rows (the score plus its ape row, as a step
// adds it), earlier ones from the compressor state as it stood before the
// pass (the current window's slots, and with overlap the previous window's),
// which nothing writes until the pass's last kernel (comp_state_after).
__device__ void compress_pass(const PrepArgs &a, float *cache, const float *kv_state, const float *score_state,
                              int y, int pos, int p0, float *cbuf, double *red)
{
    const int ratio = a.ratio, hd = a.hd, overlap = (ratio == 4), width = (1 + overlap) * hd;
    const int avail = (pos + 1) / ratio;
    if (threadIdx.x == 0) {
        a.dyn[2 * y] = avail;
        a.dyn[2 * y + 1] = avail < a.index_topk ? avail : a.index_topk;
    }
    if ((pos + 1) % ratio != 0) return;
    const int e = avail - 1, cw = p0 / ratio;
    comp_pool(cbuf, hd, overlap ? 2 * ratio : ratio, [&](int s, int c) {
        // slot s: position q, column col of its projection row (overlap:
        // the previous window's first half-width, then the current window's
        // second half-width)
        int q = e * ratio + s, col = c;
        if (overlap) {
            q = s < ratio ? (e - 1) * ratio + s : e * ratio + (s - ratio);
            col = s < ratio ? c : hd + c;
        }
        if (q < 0) return make_float2(0.0f, -INFINITY);    // before position 0: never written
        if (q >= p0) {
            const size_t r = (size_t)(q - p0) * 2 * hd + col;
            return make_float2(a.comp_in[r], __fadd_rn(a.comp_sc[r], a.ape[(size_t)(q % ratio) * width + col]));
        }
        // before the pass: the current window's slots, or the previous window's
        const int slot = (q >= cw * ratio && overlap ? ratio : 0) + q % ratio;
        return make_float2(kv_state[(size_t)slot * width + col], score_state[(size_t)slot * width + col]);
    });
    __syncthreads();
    comp_finish(cache, cbuf, a.cnorm, hd, a.rd, a.cs, a.sn, pos + 1 - ratio, a.eps, a.win + e, red);
}

// The compressor state after a prefill pass of nt tokens (p0 .. pe - 1): what
// the per-token steps leave, for every slot a later step reads before it is
// overwritten -- with overlap the previous window's slots (window pe / ratio
// - 1, when the pass closed one), then the current window's slots of the
// positions it already holds (the ones inside the pass; earlier ones are in
// place). One block.
__device__ void comp_state_after(const PrepArgs &a, float *kv_state, float *score_state, int p0, int pe)
{
    const int ratio = a.ratio, hd = a.hd, overlap = (ratio == 4), width = (1 + overlap) * hd;
    const int cw = p0 / ratio, cwn = pe / ratio;
    if (overlap && cwn > cw) {
        // window cwn - 1's positions: inside the pass, or (when it is the
        // window current before the pass) in the current slots
        for (int i = threadIdx.x; i < ratio * width; i += blockDim.x) {
            const int s = i / width, col = i - s * width, q = (cwn - 1) * ratio + s;
            float kv, sc;
            if (q >= p0) {
                const size_t r = (size_t)(q - p0) * 2 * hd + col;
                kv = a.comp_in[r];
                sc = __fadd_rn(a.comp_sc[r], a.ape[(size_t)s * width + col]);
            } else {
                kv = kv_state[(size_t)(ratio + s) * width + col];
                sc = score_state[(size_t)(ratio + s) * width + col];
            }
            kv_state[i] = kv;
            score_state[i] = sc;
        }
    }
    __syncthreads();
    const int held = pe - cwn * ratio;           // positions of window cwn already processed
    for (int i = threadIdx.x; i < held * width; i += blockDim.x) {
        const int ph = i / width, col = i - ph * width, q = cwn * ratio + ph;
        if (q < p0) continue;
        const size_t r = (size_t)(q - p0) * 2 * hd + col, dst = (size_t)((overlap ? ratio : 0) + ph) * width + col;
        kv_state[dst] = a.comp_in[r];
        score_state[dst] = __fadd_rn(a.comp_sc[r], a.ape[(size_t)ph * width + col]);
    }
}
// The attended rows of one token (src/model/dsv4_layer.c:504 and :295): the
// window newest first, then the compressed rows -- the indexer's selection
// (sel) on indexer layers, else all (pos + 1) / ratio of them -- in cache
// coordinates; -1 past the end. In a prefill pass whose first position is p0
// the window positions from p0 on are in staging rows (position q at row
// stage + q - p0), the older ones in the ring (p0 = INT_MAX: ring only).
__device__ void build_idxs(int *idxs, int nmax, int pos, int win, int has_comp, int has_idx, int take,
                           const int *sel, int p0, int stage)
{
    const int n = (pos + 1 < win) ? pos + 1 : win;
    if (!has_comp) take = 0;
    for (int i = threadIdx.x; i < nmax; i += blockDim.x) {
        int v = -1;
        if (i < n) v = (pos - i >= p0) ? stage + (pos - i - p0) : (pos - i) % win;
        else if (i < n + take) v = (has_idx ? __ldcg(sel + i - n) : i - n) + win;
        idxs[i] = v;
    }
}

// Everything between the q projections and the indexer / attention of one
// layer, one block per task (src/model/dsv4_layer.c:224-295): blocks
// [0, H) normalise and rotate a q head, block H finishes the KV row, then
// (compressing layers) one block runs the compressor step, then (indexer
// layers) ih blocks rotate the indexer's q heads, or (other layers) one block
// writes the attended row list. Every task is the whole-block code of the
// kernel it replaces, so the results are those of the separate launches.
__global__ void __launch_bounds__(256) k_attn_prep(const __grid_constant__ PrepArgs a)
{
    pdl_trigger();
    pdl_wait();
    extern __shared__ float cbuf[];     // [hd], the compressor's row
    __shared__ double red[33];
    // sequence blockIdx.y of a batch: its activations, cache and compressor
    // (pointers computed here; the argument block itself is never modified)
    const size_t y = blockIdx.y;
    float *const q = a.q + y * a.H * a.hd, *const kv = a.kv + y * a.hd, *const cache = a.cache + y * a.s_cache;
    float *const comp_kv = a.comp_kv ? a.comp_kv + y * a.s_comp : nullptr;
    float *const comp_score = a.comp_score ? a.comp_score + y * a.s_comp : nullptr;
    float *const idx_q = a.idx_q + y * a.ih * a.id;
    const float *const comp_in = a.comp_in + y * 2 * a.hd, *const comp_sc = a.comp_sc + y * 2 * a.hd;
    int *const idxs = a.idxs + y * a.nidx;
    const int pos = a.st[y].pos;
    // a prefill pass: the first token's position (its staging rows start there)
    const int p0 = a.pass_nt ? a.st[0].pos : INT_MAX;
    int b = blockIdx.x;
    if (b < a.H) {
        head_norm_rope(q + (size_t)b * a.hd, a.hd, a.rd, a.cs, a.sn, pos, 0, 1, a.eps, red);
        return;
    }
    b -= a.H;
    if (b == 0) {
        const int row = a.pass_nt ? a.stage + (int)y : pos % a.win;
        kv_finish(kv, a.kv_norm, a.hd, a.rd, a.cs, a.sn, pos, a.eps, cache + (size_t)row * a.hd, red);
        return;
    }
    b -= 1;
    if (a.has_comp) {
        if (b == 0) {
            if (!a.pass_nt) {
                compress_step(cache, comp_kv, comp_score, comp_in, comp_sc, a.ape, a.cnorm, a.ratio, a.hd,
                              a.rd, a.cs, a.sn, pos, a.eps, a.win, a.index_topk, a.dyn, cbuf, red);
            } else {
                // a prefill pass: token y's counts and (closing a window) its
                // compressed row; the state moves on after the pass
                compress_pass(a, cache, comp_kv, comp_score, (int)y, pos, p0, cbuf, red);
            }
            return;
        }
        b -= 1;
    }
    if (a.has_idx) {
        if (b < a.ih) head_norm_rope(idx_q + (size_t)b * a.id, a.id, a.rd, a.cs, a.sn, pos, 0, 0, a.eps, red);
        return;
    }
    if (b == 0)
        build_idxs(idxs, a.nidx, pos, a.win, a.has_comp, 0, a.has_comp ? (pos + 1) / a.ratio : 0, nullptr, p0,
                   a.stage);
}

// The attention index list (src/model/dsv4_layer.c:504-505 and :278-297):
// the window's ring slots of the last min(pos+1, win) positions, newest
// first, then the compressed selections (top-k order, or 0..avail-1 without
// an indexer) offset by win, then -1 up to nmax.
// One block per sequence of a batch (block b: idxs + b nmax, st[b], sel + b
// sel_stride, its counts at dyn + b dyn_stride), or per token of a prefill
// pass (stage >= 0: the pass's window rows in staging rows from stage).
__global__ void k_build_idxs(int *idxs, int nmax, const StepState *st, int win, int has_comp, int has_idx,
                             const int *dyn, const int *sel, int sel_stride, int dyn_stride, int stage)
{
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x;
    build_idxs(idxs + (size_t)b * nmax, nmax, st[b].pos, win, has_comp, has_idx,
               has_comp ? __ldcg(dyn + (size_t)b * dyn_stride + (has_idx ? 1 : 0)) : 0, sel + (size_t)b * sel_stride,
               stage >= 0 ? st[0].pos : INT_MAX, stage);
}

// The end of a prefill pass (a.pass_nt tokens): its KV rows move from the
// staging rows into the window ring (token t at slot pos_t % win; only the
// last min(nt, win) tokens are copied, earlier ones would be overwritten, so
// no slot is written twice), one block per token, and one more block moves
// the compressor state past the pass.
__global__ void k_stage_commit(const __grid_constant__ PrepArgs a)
{
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x, nt = a.pass_nt;
    if (t == nt) {
        if (a.has_comp) comp_state_after(a, a.comp_kv, a.comp_score, a.st[0].pos, a.st[nt - 1].pos + 1);
        return;
    }
    if (t < nt - a.win) return;
    const float *src = a.cache + (size_t)(a.stage + t) * a.hd;
    float *dst = a.cache + (size_t)(a.st[t].pos % a.win) * a.hd;
    for (int i = threadIdx.x; i < a.hd; i += blockDim.x) dst[i] = src[i];
}

// Argmax, first maximum (src/cli/dsv4_run.c:472-473), two stages; the second
// also advances the step state: next token = the prompt's while prompt
// remains, else the argmax; out_tokens[pos] = the argmax.
__global__ void k_argmax_part(float *pv, int *pi, const float *x, int n)
{
    pdl_trigger();
    pdl_wait();
    // sequence blockIdx.y of a batch: its logits and its kArgmaxParts partials
    pv += (size_t)blockIdx.y * kArgmaxParts;
    pi += (size_t)blockIdx.y * kArgmaxParts;
    x += (size_t)blockIdx.y * n;
    __shared__ float sv[32];
    __shared__ int si[32];
    float bv = -INFINITY;
    int bi = -1;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        if (bi < 0 || x[i] > bv) { bv = x[i]; bi = i; }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (blockDim.x >> 5); w++)
            if (si[w] >= 0 && (bi < 0 || sv[w] > bv || (sv[w] == bv && si[w] < bi))) { bv = sv[w]; bi = si[w]; }
        pv[blockIdx.x] = bv;
        pi[blockIdx.x] = bi;
    }
}

// The best (value, index) of pv[i * stride], pi[i * stride], i < nparts, by
// one warp: each lane the best of its strided share, then the same comparison
// (larger value, ties to the lower index) across lanes.
__device__ __forceinline__ void argmax_warp(float &bv, int &bi, const float *pv, const int *pi, int nparts,
                                            int stride)
{
    bv = -INFINITY;
    bi = -1;
    for (int i = threadIdx.x; i < nparts; i += 32) {
        const float v = ld_act(pv + (size_t)i * stride);
        const int ix = __ldcg(pi + (size_t)i * stride);
        if (ix >= 0 && (bi < 0 || v > bv || (v == bv && ix < bi))) { bv = v; bi = ix; }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
    }
}

__global__ void k_argmax_final(StepState *st, int *out_tokens, const float *pv, const int *pi, int nparts,
                               int stride, const int *prompt, int n_prompt, unsigned *stepseq, int seq_tokens)
{
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x >= 32) return;
    // sequence blockIdx.x of a batch: its state, its token rows (seq_tokens
    // apart) and its partials
    const int sq = blockIdx.x;
    st += sq;
    out_tokens += (size_t)sq * seq_tokens;
    prompt += (size_t)sq * seq_tokens;
    pv += (size_t)sq * kArgmaxParts;
    pi += (size_t)sq * kArgmaxParts;
    if (sq != 0) stepseq = nullptr;
    float bv;
    int bi;
    argmax_warp(bv, bi, pv, pi, nparts, stride);
    if (threadIdx.x != 0) return;
    const int pos = st->pos;
    out_tokens[pos] = bi;
    const int next = pos + 1;
    st->token = (next < n_prompt) ? prompt[next] : bi;
    st->pos = next;
    if (stepseq) *stepseq += 1u;          // sharded: the exchanges' step count
}

// A rank's best pair of its vocabulary slice, the index made global:
// pair = {value, index bits}.
__global__ void k_argmax_pair(float *pair, const float *pv, const int *pi, int nparts, int offset)
{
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x >= 32) return;
    float bv;
    int bi;
    argmax_warp(bv, bi, pv, pi, nparts, 1);
    if (threadIdx.x == 0) {
        pair[0] = bv;
        pair[1] = __int_as_float(bi >= 0 ? bi + offset : -1);
    }
}

}  // namespace dsv4b

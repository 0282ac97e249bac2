// moe.cu - the routed-expert FFN for one token, on the device.
//
// Restates moe() (src/model/dsv4_layer.c:369-484): router GEMV, scoring and
// top-k (src/core/dsv4_ops.c:102-141), each selected expert's w1/w3 GEMV,
// SwiGLU (dsv4_ops.c:60-78), w2 GEMV into a per-k accumulator, the weighted
// sum strictly in k order, then the shared expert added unweighted. The
// experts are picked on the device (sel[] written by the router kernel and
// read by the GEMVs through a device pointer table), so a decode step never
// waits on the host between routing and the expert matmuls.
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "moe.h"

namespace dsv4b {

// Router scoring and selection (dsv4_ops.c:102-141, with sigmoid from
// tools/dsv4_ref.py:64-93). One block. fixed != nullptr means hash routing:
// the experts are given (tid2eid row), the weights still come from scores.
// A batch: block b routes token b (logits, sel_out, w_out s_ms apart; its
// token id tok_stride ints after token b - 1's).
__global__ void k_route(const float *logits, const float *bias, const int *fixed,
                        const int64_t *tid2eid, const int *token, int n, int topk,
                        float route_scale, int score_func, int *sel_out, float *w_out, long s_ms, int tok_stride)
{
    pdl_trigger();
    pdl_wait();
    logits += blockIdx.x * s_ms;
    sel_out += blockIdx.x * s_ms;
    w_out += blockIdx.x * s_ms;
    if (token) token += (size_t)blockIdx.x * tok_stride;
    __shared__ float orig[kMoeMaxExperts], sc[kMoeMaxExperts];
    __shared__ int chosen[kMoeMaxTopk];
    const int tid = threadIdx.x, nthr = blockDim.x;
    for (int e = tid; e < n; e += nthr) {
        const float l = logits[e];
        float o;
        if (score_func == 2) o = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-l)));
        else o = sqrtf((l > 20.0f) ? l : log1pf(expf(l)));
        orig[e] = o;
        sc[e] = bias ? __fadd_rn(o, bias[e]) : o;
    }
    __syncthreads();
    if (fixed || tid2eid) {
        if (tid < topk) chosen[tid] = fixed ? fixed[tid] : (int)tid2eid[(long)token[0] * topk + tid];
    } else if (tid < 32) {
        // topk rounds of warp argmax: value descending, ties to the lower
        // index -- the order of the reference's repeated-argmax selection.
        // Lane l holds experts l + 32 i in registers and its current best;
        // the round's winner drops its candidate (to -inf: scores are finite)
        // and rescans its own.
        constexpr int PER = kMoeMaxExperts / 32;
        float v[PER];
#pragma unroll
        for (int i = 0; i < PER; i++) {
            const int e = tid + 32 * i;
            v[i] = e < n ? sc[e] : -INFINITY;
        }
        auto local_best = [&](float &bv, int &bi) {
            bv = -INFINITY;
            bi = -1;
#pragma unroll
            for (int i = 0; i < PER; i++)
                if (v[i] != -INFINITY && (bi < 0 || v[i] > bv)) { bv = v[i]; bi = tid + 32 * i; }
        };
        float lv;
        int li;
        local_best(lv, li);
        for (int k = 0; k < topk; k++) {
            float bv = lv;
            int bi = li;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
            }
            if (tid == 0) chosen[k] = bi;
            if (bi >= 0 && (bi & 31) == tid) {
#pragma unroll
                for (int i = 0; i < PER; i++)
                    if (tid + 32 * i == bi) v[i] = -INFINITY;
                local_best(lv, li);
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        float wts[kMoeMaxTopk];
        double sum = 0.0;
        for (int k = 0; k < topk; k++) { wts[k] = orig[chosen[k]]; sum += (double)wts[k]; }
        const float inv = (sum != 0.0) ? __fdiv_rn(1.0f, (float)sum) : 0.0f;
        for (int k = 0; k < topk; k++) {
            w_out[k] = __fmul_rn(__fmul_rn(wts[k], inv), route_scale);
            sel_out[k] = chosen[k];
        }
    }
}

// The union of a batch's experts, in groups: the (token, slot) pairs are
// ordered by (expert, token, slot), each expert's run is cut into groups of
// at most `chunk` pairs, and group g is written as groups[5 g] = its size,
// groups[5 g + 1 ..] = (t << 8) | k; the slots after the last group get size
// 0. A routed item per slot then streams and decodes its expert once for
// every token of its group. One block; n = nseq topk <= 1024.
__global__ void k_moe_group(const int *sel, long s_ms, int nseq, int topk, int chunk, int *groups)
{
    pdl_trigger();
    pdl_wait();
    __shared__ int es[1024], ord[1024];
    __shared__ int s_ng;
    const int n = nseq * topk;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int t = i / topk, k = i - t * topk;
        es[i] = __ldcg(sel + (size_t)t * s_ms + k);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int e = es[i];
        int r = 0;
        for (int j = 0; j < n; j++) r += (es[j] < e) || (es[j] == e && j < i);
        ord[r] = i;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int ng = 0, run = 0, prev = -1;
        for (int r = 0; r < n; r++) {
            const int i = ord[r], e = es[i];
            if (e != prev || run == chunk) {      // a new group
                ng++;
                run = 0;
                prev = e;
            }
            const int t = i / topk;
            groups[(size_t)(ng - 1) * 5 + 1 + run] = (t << 8) | (i - t * topk);
            groups[(size_t)(ng - 1) * 5] = ++run;
        }
        s_ng = ng;
    }
    __syncthreads();
    for (int g = s_ng + threadIdx.x; g < n; g += blockDim.x) groups[(size_t)g * 5] = 0;
}

// out[i] = sum_k w[k] * acc[k][i] in k order, each product and sum rounded
// separately (dsv4_layer.c:471-475), then + shared[i] (:479-483).
__global__ void k_combine(float *out, const float *acc, const float *w, int topk, int hidden,
                          const float *shared)
{
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= hidden) return;
    float o = 0.0f;
    for (int k = 0; k < topk; k++) o = __fadd_rn(o, __fmul_rn(w[k], acc[(size_t)k * hidden + i]));
    if (shared) o = __fadd_rn(o, shared[i]);
    out[i] = o;
}

int moe_forward(const MoeLayer &L, const MoeScratch &S, float *out, const float *x,
                const int *token, cudaStream_t st, bool combine, const Exch *ex, int nseq, long s_ms, long s_x,
                int tok_stride, int *perm)
{
    const int H = L.hidden, I = L.inter, K = L.topk;
    PdlChain chain;
    if (K < 1 || K > kMoeMaxTopk || L.n_experts > kMoeMaxExperts || nseq < 1) return -1;
    if (nseq > 1 && (combine || ex)) return -1;          // a batch folds its combine into the next mHC
    if (nseq == 1) {
        s_ms = 0;
        s_x = H;
    }
    // router: one item per token, each the batch-1 arithmetic
    if (gemv(L.gate.wdt, S.logits, nseq > 1 ? s_ms : L.n_experts, x, s_x, L.gate.w, L.gate.s, L.n_experts, H,
             L.gate.blk_r, L.gate.blk_c, nseq, st, L.gate.f16s != 0))
        return -1;
    launch(k_route, dim3(nseq), dim3(256), 0, st, S.logits, L.bias, L.fixed, L.tid2eid, token, L.n_experts, K,
           L.route_scale, L.score_func, S.sel, S.wts, s_ms, tok_stride);
    const int Is = L.has_shared ? L.inter_shared : 0;
    // a batch on the tensor-core path: the routed items in expert order (the
    // order is picked on the device; every item's arithmetic is unchanged)
    const bool sorted = nseq > 1 && perm && nseq * K <= 1024 &&
                        gemv_mma_shape(L.efmt, H, L.eblk_r, L.eblk_c, L.ef16s != 0) &&
                        gemv_mma_shape(L.efmt, I, L.eblk_r, L.eblk_c, L.ef16s != 0);
    // tokens per group: what both the gate / up and the down items can carry
    int chunk = 1;
    if (sorted) {
        GemvItem u, dn;
        if (!gemv_item(u, L.efmt, nullptr, nullptr, I, H, L.eblk_r, L.eblk_c, x, S.h, L.ef16s != 0) ||
            !gemv_item(dn, L.efmt, nullptr, nullptr, H, I, L.eblk_r, L.eblk_c, S.h, S.acc, L.ef16s != 0))
            return -1;
        u.pair = 1;
        // two tokens keep two blocks per SM (four need the one-block budget)
        const int cu = gemv_item_tokens(u, 2, 0, 0), cd = gemv_item_tokens(dn, 2, 0, 0);
        chunk = cu < cd ? cu : cd;
        launch(k_moe_group, dim3(1), dim3(256), 0, st, S.sel, s_ms, nseq, K, chunk, perm);
    }
    // the items of one stage (every token's selected experts, then its shared
    // expert), launched kGemvMaxItems at a time: a launch's grouping never
    // changes an item's arithmetic
    std::vector<GemvItem> items;
    auto flush = [&]() -> int {
        for (size_t i0 = 0; i0 < items.size(); i0 += kGemvMaxItems) {
            const int n = (int)std::min<size_t>(kGemvMaxItems, items.size() - i0);
            if (gemv_group(items.data() + i0, n, st)) return -1;
        }
        items.clear();
        return 0;
    };
    // gate / up of every selected expert and the shared one, SwiGLU in the
    // epilogue: h[k] = swiglu(w1 x, w3 x) (dsv4_layer.c:199-206)
    if (sorted) {
        for (int j = 0; j < nseq * K; j++) {
            GemvItem it;
            if (!gemv_item(it, L.efmt, nullptr, nullptr, I, H, L.eblk_r, L.eblk_c, x, S.h, L.ef16s != 0) || !it.mma)
                return -1;
            it.wtab = L.w1tab; it.stab = L.s1tab;
            it.w2tab = L.w3tab; it.s2tab = L.s3tab;
            it.sel = S.sel; it.slot = j;
            it.perm = perm; it.xs = (int)s_x; it.xk = 0; it.ys = (int)s_ms; it.yk = I; it.ss = (int)s_ms;
            it.nt = chunk;
            it.pair = 1; it.limit = L.swiglu_limit;
            items.push_back(it);
        }
    }
    for (int b = 0; b < nseq; b++) {
        const float *xb = x + (size_t)b * s_x;
        float *hb = S.h + (size_t)b * s_ms;
        const int *selb = S.sel + (size_t)b * s_ms;
        for (int k = 0; k < K && !sorted; k++) {
            GemvItem it;
            if (!gemv_item(it, L.efmt, nullptr, nullptr, I, H, L.eblk_r, L.eblk_c, xb, hb + (size_t)k * I,
                           L.ef16s != 0))
                return -1;
            it.wtab = L.w1tab; it.stab = L.s1tab;
            it.w2tab = L.w3tab; it.s2tab = L.s3tab;
            it.sel = selb; it.slot = k;
            it.pair = 1; it.limit = L.swiglu_limit;
            items.push_back(it);
        }
    }
    // the shared expert: a batch's tokens several to an item
    for (int b = 0; Is && b < nseq;) {
        GemvItem it;
        if (!gemv_item(it, L.sh[0].wdt, L.sh[0].w, L.sh[0].s, Is, H, L.sh[0].blk_r, L.sh[0].blk_c,
                       x + (size_t)b * s_x, S.h + (size_t)b * s_ms + (size_t)K * I, L.sh[0].f16s && L.sh[1].f16s) ||
            L.sh[1].wdt != L.sh[0].wdt)
            return -1;
        it.W2 = L.sh[1].w; it.S2 = L.sh[1].s;
        it.pair = 1; it.limit = L.swiglu_limit;
        b += gemv_item_tokens(it, nseq - b, s_x, s_ms);
        items.push_back(it);
    }
    if (flush()) return -1;
    // down projections into the per-k accumulators
    if (sorted) {
        for (int j = 0; j < nseq * K; j++) {
            GemvItem it;
            if (!gemv_item(it, L.efmt, nullptr, nullptr, H, I, L.eblk_r, L.eblk_c, S.h, S.acc, L.ef16s != 0) ||
                !it.mma)
                return -1;
            it.wtab = L.w2tab; it.stab = L.s2tab;
            it.sel = S.sel; it.slot = j;
            it.perm = perm; it.xs = (int)s_ms; it.xk = I; it.ys = (int)s_ms; it.yk = H; it.ss = (int)s_ms;
            it.nt = chunk;
            items.push_back(it);
        }
    }
    for (int b = 0; b < nseq; b++) {
        const float *hb = S.h + (size_t)b * s_ms;
        float *accb = S.acc + (size_t)b * s_ms;
        const int *selb = S.sel + (size_t)b * s_ms;
        for (int k = 0; k < K && !sorted; k++) {
            GemvItem it;
            if (!gemv_item(it, L.efmt, nullptr, nullptr, H, I, L.eblk_r, L.eblk_c, hb + (size_t)k * I,
                           accb + (size_t)k * H, L.ef16s != 0))
                return -1;
            it.wtab = L.w2tab; it.stab = L.s2tab;
            it.sel = selb; it.slot = k;
            items.push_back(it);
        }
    }
    for (int b = 0; Is && b < nseq;) {
        GemvItem it;
        if (!gemv_item(it, L.sh[2].wdt, L.sh[2].w, L.sh[2].s, H, Is, L.sh[2].blk_r, L.sh[2].blk_c,
                       S.h + (size_t)b * s_ms + (size_t)K * I, S.acc + (size_t)b * s_ms + (size_t)K * H,
                       L.sh[2].f16s != 0))
            return -1;
        b += gemv_item_tokens(it, nseq - b, s_ms, s_ms);
        items.push_back(it);
    }
    if (flush()) return -1;
    float *accs = S.acc + (size_t)K * H;
    // sharded: every rank holds a slice of each expert's inter dimension, so
    // its outputs are partial sums over that slice; add them up across ranks
    if (ex && xreduce_sum(*ex, S.acc, (size_t)(K + (Is ? 1 : 0)) * H, st)) return -1;
    if (combine)
        launch(k_combine, dim3((H + 255) / 256), dim3(256), 0, st, out, S.acc, S.wts, K, H, Is ? accs : nullptr);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

size_t moe_scratch_floats(int hidden, int inter, int inter_shared, int n_experts, int topk)
{
    const size_t im = (size_t)topk * inter + inter_shared;
    return (size_t)n_experts + 3 * im + (size_t)(topk + 1) * hidden + 2 * kMoeMaxTopk;
}

void moe_scratch_carve(MoeScratch &S, float *base, int hidden, int inter, int inter_shared, int n_experts,
                       int topk)
{
    const size_t im = (size_t)topk * inter + inter_shared;
    float *p = base;
    S.logits = p; p += n_experts;
    S.g = p; p += im;
    S.u = p; p += im;
    S.h = p; p += im;
    S.acc = p; p += (size_t)(topk + 1) * hidden;
    S.wts = p; p += kMoeMaxTopk;
    S.sel = reinterpret_cast<int *>(p);
}

}  // namespace dsv4b

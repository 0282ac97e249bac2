// model.cu - whole-token decode with every weight resident in HBM.
//
// One decode token of src/cli/dsv4_run.c:444-483 (embed, every
// dsv4_layer_forward, hc_head, final norm, LM head, argmax) as a fixed
// sequence of device launches: the GEMVs of gemv.cu, moe_forward of moe.cu,
// the sparse-MLA kernels of mla.cu and the support ops of model_kernels.cu.
// Nothing in the sequence depends on the host: the position and token live in
// a device StepState that the last kernel advances, so the sequence is
// captured once into a CUDA graph and replayed for every position. The same
// sequence serves a batch of sequences (one row each) and a prefill pass of
// one sequence's prompt tokens (dsv4_run.c:391-442, one row per token; see
// attn_core for how the pass keeps each token's view of the caches).
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <utility>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "mla.h"
#include "model.h"
#include "../../include/dsv4_b200.h"

namespace dsv4b {

struct DevLayer {
    float *attn_norm, *ffn_norm, *sink, *q_norm, *kv_norm;
    DevMat wq_a, wq_b, wkv, wo_a, wo_b;
    int ratio, has_comp, has_idx, coff;
    float *ape, *cnorm;
    DevMat cwkv, cwgate, iwq_b, iwproj;
    float *hca_fn, *hca_base, *hca_scale, *hcf_fn, *hcf_base, *hcf_scale;
    MoeLayer moe;
    float *kv_cache, *comp_kv, *comp_score;
    int *dyn;
    // cache rows: the window ring, the compressed rows, then (a one-sequence
    // model) a prefill pass's staging rows from stage_row
    size_t kv_rows, comp_n;
    int stage_row;
};

}  // namespace dsv4b

struct dsv4b_model {
    DSV4Cfg c;
    int ratios[DSV4_MAX_LAYERS];
    int max_pos, nidx, ncomp4;
    std::vector<dsv4b::DevLayer> L;
    const void *embed;
    int emb_wdt;
    dsv4b::DevMat head;
    float *norm, *hch_fn, *hch_base, *hch_scale;
    float *cs_d, *sn_d, *cs_c, *sn_c;
    float *h, *resid, *x1, *blk, *post, *comb, *mixes, *qr, *q, *kv, *o, *ogrp;
    float *comp_in, *comp_sc, *idx_q, *idx_w, *idx_scores, *logits, *xh, *am_pv;
    int *idxs, *isel, *am_pi, *prompt, *out_tokens;
    void *attn_part;
    double *hc_part;
    unsigned *hc_cnt;
    dsv4b::MoeScratch ms;
    dsv4b::StepState *st;
    // sharding: rank of world GPUs; comm is the NCCL communicator (null on one
    // GPU); am_pair / am_gather hold the LM-head argmax exchange
    int rank, world;
    void *comm, *peer;
    unsigned *stepseq;         // steps done (device; advanced by the last kernel)
    double *ix_terms;          // the head-split indexer's scratch
    unsigned *ix_count;
    int nx, xcall;             // exchanges per step; the next one's index
    float *am_pair, *am_gather;
    int n_prompt;
    // a batch: nseq sequences decoded in lockstep (the same positions), each
    // with its own activations, caches, step state and tokens; per-sequence
    // buffers are packed (sequence b at b times the one-sequence size), the
    // MoE scratch s_ms floats apart
    int nseq;
    long s_ms;
    int *moe_perm;             // a batch's expert groups (5 ints per slot, k_moe_group)
    // activation rows: nseq, or on a one-sequence model the tokens of a
    // prefill pass (pst holds their step states)
    int cap;
    dsv4b::StepState *pst;
    int *pdyn;                 // a prefill pass's per-token compressed-row counts (2 ints each)
    int ix_rows;               // rows of the indexer's head-split scratch (ix_terms / ix_count)
    // prefill passes as graphs, one per (tokens, last) shape: a shape runs
    // eagerly the first time (which also sets every kernel attribute), is
    // captured the second, replayed after; pf_kernels counts the kernels the
    // last prefill launched (-1 when a pass ran eagerly)
    struct PassGraph {
        int key, kernels;
        cudaGraph_t graph;
        cudaGraphExec_t exec;
    };
    std::vector<PassGraph> pgraphs;
    std::vector<int> pseen;
    int pf_kernels;
    std::vector<void *> allocs;
    cudaStream_t stream;
    cudaGraph_t graph;
    cudaGraphExec_t exec;
    int graphed;
};

namespace dsv4b {

static void *dalloc(dsv4b_model *m, size_t bytes)
{
    void *p = nullptr;
    if (cudaMalloc(&p, bytes ? bytes : 16) != cudaSuccess) return nullptr;
    m->allocs.push_back(p);
    return p;
}

static void *dcopy(dsv4b_model *m, const void *host, size_t bytes, bool *ok)
{
    if (!*ok) return nullptr;
    void *p = dalloc(m, bytes);
    if (!p || (host && cudaMemcpy(p, host, bytes, cudaMemcpyHostToDevice) != cudaSuccess)) {
        *ok = false;
        return nullptr;
    }
    return p;
}

static size_t qmat_sbytes(const DSV4QMat &q)
{
    if (q.wdt < DSV4_WFP8) return 0;
    return (size_t)((q.rows + q.blk_r - 1) / q.blk_r) * ((q.cols + q.blk_c - 1) / q.blk_c);
}

static DevMat up_mat(dsv4b_model *m, const DSV4QMat &q, bool *ok)
{
    DevMat d = {};
    d.wdt = q.wdt;
    d.rows = q.rows;
    d.cols = q.cols;
    d.blk_r = q.blk_r;
    d.blk_c = q.blk_c;
    if (!q.w) { *ok = false; return d; }
    d.w = (const uint8_t *)dcopy(m, q.w, row_bytes(q.wdt, q.cols) * q.rows, ok);
    if (q.wdt >= DSV4_WFP8) d.s = (const uint8_t *)dcopy(m, q.s, qmat_sbytes(q), ok);
    d.f16s = q.wdt == DSV4_WFP4 && q.s && fp4_scales_f16((const uint8_t *)q.s, qmat_sbytes(q));
    return d;
}

static float *up_f32(dsv4b_model *m, const float *p, size_t n, bool *ok)
{
    return (float *)dcopy(m, p, n * 4, ok);
}

// RoPE cos/sin tables (src/core/dsv4_rope.c:48-99), computed on the host in
// double exactly as the reference does, then copied to the device.
static void rope_table(float *cs, float *sn, int dim, int seqlen, int orig, double base, double factor,
                       double beta_fast, double beta_slow)
{
    const int half = dim / 2;
    std::vector<double> f(half);
    for (int i = 0; i < half; i++) f[i] = 1.0 / pow(base, (double)(2 * i) / (double)dim);
    if (orig > 0) {
        const double twopi = 2.0 * 3.14159265358979323846;
        const double lo_d = (double)dim * log((double)orig / (beta_fast * twopi)) / (2.0 * log(base));
        const double hi_d = (double)dim * log((double)orig / (beta_slow * twopi)) / (2.0 * log(base));
        int lo = (int)floor(lo_d), hi = (int)ceil(hi_d);
        if (lo < 0) lo = 0;
        if (hi > dim - 1) hi = dim - 1;
        double mn = (double)lo, mx = (double)hi;
        if (mn == mx) mx += 0.001;
        for (int i = 0; i < half; i++) {
            double ramp = ((double)i - mn) / (mx - mn);
            if (ramp < 0.0) ramp = 0.0;
            if (ramp > 1.0) ramp = 1.0;
            const double smooth = 1.0 - ramp;
            f[i] = f[i] / factor * (1.0 - smooth) + f[i] * smooth;
        }
    }
    for (int t = 0; t < seqlen; t++)
        for (int i = 0; i < half; i++) {
            const double th = (double)t * f[i];
            cs[(size_t)t * half + i] = (float)cos(th);
            sn[(size_t)t * half + i] = (float)sin(th);
        }
}

// Allocate the activations, state and tables every model needs.
static bool alloc_common(dsv4b_model *m)
{
    const DSV4Cfg &c = m->c;
    bool ok = true;
    const int hc = c.hc_mult, d = c.hidden, hd = c.head_dim, win = c.sliding_window;
    const int half = c.qk_rope / 2;
    std::vector<float> cs((size_t)m->max_pos * half), sn((size_t)m->max_pos * half);
    rope_table(cs.data(), sn.data(), c.qk_rope, m->max_pos, 0, c.rope_theta, c.yarn_factor, c.yarn_beta_fast,
               c.yarn_beta_slow);
    m->cs_d = (float *)dcopy(m, cs.data(), cs.size() * 4, &ok);
    m->sn_d = (float *)dcopy(m, sn.data(), sn.size() * 4, &ok);
    rope_table(cs.data(), sn.data(), c.qk_rope, m->max_pos, c.yarn_orig_ctx, c.compress_rope_theta,
               c.yarn_factor, c.yarn_beta_fast, c.yarn_beta_slow);
    m->cs_c = (float *)dcopy(m, cs.data(), cs.size() * 4, &ok);
    m->sn_c = (float *)dcopy(m, sn.data(), sn.size() * 4, &ok);
    // the attention index list: window + the most compressed rows any layer adds
    int extra = 0;
    m->ncomp4 = 1;
    for (int L = 0; L < c.n_layers; L++) {
        const int r = m->ratios[L];
        if (r == 4) m->ncomp4 = m->max_pos / 4 + 1;
        const int add = r == 0 ? 0 : (r == 4 ? c.index_topk : m->max_pos / r + 1);
        if (add > extra) extra = add;
    }
    m->nidx = win + extra;
    const size_t big = (size_t)(d > c.q_lora ? d : c.q_lora);
    // B: sequences (caches, step states, tokens); R: activation rows
    const size_t B = (size_t)m->nseq, R = (size_t)m->cap;
    auto F = [&](size_t n) { return (float *)dcopy(m, nullptr, n * 4, &ok); };
    m->h = F(R * hc * d);
    m->resid = F(R * hc * d);
    m->x1 = F(R * d);
    m->blk = F(R * d);
    m->post = F(R * DSV4B_MAX_HC);
    m->comb = F(R * DSV4B_MAX_HC * DSV4B_MAX_HC);
    m->mixes = F((2 + DSV4B_MAX_HC) * DSV4B_MAX_HC);
    m->qr = F(R * big);
    m->q = F(R * c.n_heads * hd);
    m->kv = F(R * hd);
    m->o = F(R * c.n_heads * hd);
    m->ogrp = F(R * c.o_groups * c.o_lora);
    m->comp_in = F(R * 2 * hd);
    m->comp_sc = F(R * 2 * hd);
    m->idx_q = F(R * c.index_n_heads * c.index_head_dim);
    m->idx_w = F(R * c.index_n_heads);
    m->idx_scores = F(R * m->ncomp4);
    // the head-split indexer's terms for up to R rows, within 256 MB (a
    // prefill pass scores its tokens in groups of ix_rows)
    const size_t ix_row = (size_t)m->ncomp4 * c.index_n_heads * 8;
    size_t ixr = (256u << 20) / (ix_row ? ix_row : 1);
    ixr = ixr < B ? B : (ixr > R ? R : ixr);
    m->ix_rows = (int)ixr;
    m->ix_terms = (double *)dcopy(m, nullptr, ixr * ix_row, &ok);
    m->ix_count = (unsigned *)dcopy(m, nullptr, ixr * ((m->ncomp4 + 31) / 32) * 4, &ok);
    if (ok && cudaMemset(m->ix_count, 0, ixr * ((m->ncomp4 + 31) / 32) * 4) != cudaSuccess) ok = false;
    m->pdyn = (int *)dcopy(m, nullptr, R * 2 * 4, &ok);
    m->logits = F(B * c.vocab);
    m->xh = F(R * d);
    m->am_pv = F(B * kArgmaxParts);
    m->am_pair = F(2);
    m->stepseq = (unsigned *)dcopy(m, nullptr, 4, &ok);
    if (ok && cudaMemset(m->stepseq, 0, 4) != cudaSuccess) ok = false;
    m->nx = 2 * c.n_layers;
    m->am_gather = F(2 * 64);
    m->am_pi = (int *)dcopy(m, nullptr, B * kArgmaxParts * 4, &ok);
    m->idxs = (int *)dcopy(m, nullptr, R * m->nidx * 4, &ok);
    m->isel = (int *)dcopy(m, nullptr, R * (c.index_topk > 0 ? c.index_topk : 1) * 4, &ok);
    m->prompt = (int *)dcopy(m, nullptr, B * m->max_pos * 4, &ok);
    m->out_tokens = (int *)dcopy(m, nullptr, B * m->max_pos * 4, &ok);
    m->st = (StepState *)dcopy(m, nullptr, B * sizeof(StepState), &ok);
    m->pst = (StepState *)dcopy(m, nullptr, R * sizeof(StepState), &ok);
    m->attn_part = dcopy(m, nullptr, attn_part_bytes(c.n_heads, hd, m->nidx, (int)R), &ok);
    m->hc_part = (double *)dcopy(m, nullptr, R * kHcPreBlocks * (kHcPreMixMax + 1) * 8, &ok);
    m->hc_cnt = (unsigned *)dcopy(m, nullptr, R * 4, &ok);
    if (ok && cudaMemset(m->hc_cnt, 0, R * 4) != cudaSuccess) ok = false;
    const int inter_s = c.moe_inter * c.n_shared;
    const size_t nf = moe_scratch_floats(d, c.moe_inter, inter_s, c.n_experts, c.topk);
    m->s_ms = (long)((nf + kMoeMaxTopk + 63) & ~(size_t)63);
    m->moe_perm = (int *)dcopy(m, nullptr, R * kMoeMaxTopk * 5 * 4, &ok);
    float *msb = F(R * m->s_ms);
    if (ok) moe_scratch_carve(m->ms, msb, d, c.moe_inter, inter_s, c.n_experts, c.topk);
    // a one-sequence model's prefill pass writes its KV rows to staging rows
    // at the end of each cache (the ring is read by the pass's own tokens)
    const size_t stage = (m->nseq == 1 && R > 1) ? R : 0;
    for (int L = 0; L < c.n_layers && ok; L++) {
        DevLayer &l = m->L[L];
        l.ratio = m->ratios[L];
        l.coff = l.ratio == 4 ? 2 : 1;
        const size_t ncomp = l.ratio ? (size_t)(m->max_pos / l.ratio + 1) : 0;
        l.stage_row = (int)(win + ncomp);
        l.kv_rows = (size_t)win + ncomp + stage;
        l.kv_cache = F(B * l.kv_rows * hd);
        l.comp_n = l.ratio ? (size_t)l.coff * l.ratio * l.coff * hd : 0;
        l.comp_kv = l.comp_n ? F(B * l.comp_n) : nullptr;
        l.comp_score = l.comp_n ? F(B * l.comp_n) : nullptr;
        l.dyn = (int *)dcopy(m, nullptr, 8, &ok);
    }
    return ok;
}

__global__ void k_fill(float *p, size_t n, float v)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) p[i] = v;
}

// Empty caches and compressor windows (score -inf: an unfilled slot must
// contribute nothing, src/model/dsv4_layer.c:100-106).
static int reset_state(dsv4b_model *m)
{
    const size_t B = (size_t)m->nseq;
    for (DevLayer &l : m->L) {
        DSV4B_CUDA_OK(cudaMemsetAsync(l.kv_cache, 0, B * l.kv_rows * m->c.head_dim * 4, m->stream));
        if (l.comp_n) {
            DSV4B_CUDA_OK(cudaMemsetAsync(l.comp_kv, 0, B * l.comp_n * 4, m->stream));
            k_fill<<<64, 256, 0, m->stream>>>(l.comp_score, B * l.comp_n, -INFINITY);
        }
        DSV4B_CUDA_OK(cudaMemsetAsync(l.dyn, 0, 8, m->stream));
    }
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

static int G(const DevMat &w, float *y, const float *x, cudaStream_t st)
{
    return gemv(w.wdt, y, w.rows, x, w.cols, w.w, w.s, w.rows, w.cols, w.blk_r, w.blk_c, 1, st, w.f16s != 0);
}

// x1 = RMSNorm(mHC pre-mix of h) with the sub-layer's norm weights.
// A grouped GEMV launch under construction; shapes the streaming kernel
// cannot take run on their own at once.
struct Grp {
    GemvItem it[kGemvMaxItems];
    int n = 0, rc = 0;
};

// nseq tokens (a batch: token b's x at x + b xs, its y at y + b ys), as
// items of up to four tokens where the matrix runs on the tensor cores (one
// weight stream per item), every token's arithmetic that of a batch-1 call;
// a full group is launched and a new one begun.
static void grp_add(Grp &g, const DevMat &w, const float *x, float *y, cudaStream_t st, int nseq = 1, long xs = 0,
                    long ys = 0)
{
    for (int b = 0; b < nseq;) {
        const float *xb = x + (size_t)b * xs;
        float *yb = y + (size_t)b * ys;
        if (g.n == kGemvMaxItems) {
            g.rc |= gemv_group(g.it, g.n, st);
            g.n = 0;
        }
        if (gemv_item(g.it[g.n], w.wdt, w.w, w.s, w.rows, w.cols, w.blk_r, w.blk_c, xb, yb, w.f16s != 0)) {
            // a batch: several tokens per item where the matrix takes them
            b += gemv_item_tokens(g.it[g.n], nseq - b, xs, ys);
            g.n++;
        } else {
            g.rc |= G(w, yb, xb, st);
            b++;
        }
    }
}

static int grp_run(Grp &g, cudaStream_t st) { return g.rc | gemv_group(g.it, g.n, st); }

// What the next mHC launch finishes before it mixes: nothing (the embedding),
// an attention output in m->blk, or an MoE's per-expert outputs (its combine).
struct Pending {
    int kind;                 // 0 none, 1 blk, 2 MoE accumulators
    const MoeLayer *moe;
};

static bool hc_fused(const DSV4Cfg &c)
{
    const int hc = c.hc_mult, n = hc * c.hidden;
    return (2 + hc) * hc <= kHcPreMixMax && c.hidden % 4 == 0 && c.hidden <= 256 * 4 * kHcPreYPT && n % 256 == 0 &&
           n / 256 <= kHcPreBlocks;
}

// The post-mix of the pending sub-layer (hin -> hout, then swapped) and the
// pre-mix of the next one into y (x1, or the head's xh when head is set), for
// the rows activation rows (a batch's sequences or a prefill pass's tokens).
static void hc_step(dsv4b_model *m, Pending &p, float *&hin, float *&hout, const float *fn, const float *base,
                    const float *scale, const float *norm, bool head, float *y, cudaStream_t st, int rows)
{
    const DSV4Cfg &c = m->c;
    const int hc = c.hc_mult, mix = (2 + hc) * hc, n = hc * c.hidden, wide = n;
    if (hc_fused(c)) {
        HcPreArgs a = {};
        a.y = y;
        a.post = head ? nullptr : m->post;
        a.comb = head ? nullptr : m->comb;
        a.x = hin;
        if (p.kind) {
            a.xout = hout;
            a.post_in = m->post;
            a.comb_in = m->comb;
            if (p.kind == 1) {
                a.blk = m->blk;
            } else {
                a.acc = m->ms.acc;
                a.wts = m->ms.wts;
                a.topk = p.moe->topk;
                a.accs = (p.moe->has_shared && p.moe->inter_shared) ? m->ms.acc + (size_t)p.moe->topk * c.hidden
                                                                       : nullptr;
            }
        }
        a.fn = fn;
        a.scale = scale;
        a.base = base;
        a.norm_w = norm;
        a.part = m->hc_part;
        a.count = m->hc_cnt;
        a.hc = hc;
        a.hidden = c.hidden;
        a.iters = c.hc_sinkhorn_iters;
        a.nmix = head ? hc : mix;
        a.hc_eps = c.hc_eps;
        a.rms_eps = c.rms_eps;
        a.s_ms = m->s_ms;
        if (rows > 1) {
            launch(k_hc_part_batch, dim3(n / 256, rows), dim3(288), 0, st, a);
            launch(k_hc_tail_batch, dim3(rows), dim3(288), 0, st, a);
        } else {
            launch(k_hc_pre, dim3(n / 256), dim3(288), 0, st, a);
        }
        if (p.kind) std::swap(hin, hout);
        p.kind = 0;
        return;
    }
    // unfused: the MoE was combined into m->blk by moe_forward
    if (p.kind) {
        launch(k_hc_post, dim3((wide + 255) / 256), dim3(256), 0, st, hout, m->blk, hin, m->post, m->comb, hc,
               c.hidden);
        std::swap(hin, hout);
        p.kind = 0;
    }
    if (head) {
        launch(k_hc_mix, dim3(hc), dim3(256), 0, st, m->mixes, fn, hin, n, c.rms_eps);
        launch(k_hc_head_finish, dim3(1), dim3(256), 0, st, y, m->mixes, hin, scale, base, hc, c.hidden, c.hc_eps);
    } else {
        launch(k_hc_mix, dim3(mix), dim3(256), 0, st, m->mixes, fn, hin, n, c.rms_eps);
        launch(k_hc_finish, dim3(1), dim3(256), 0, st, y, m->post, m->comb, m->mixes, hin, scale, base, hc, c.hidden,
               c.hc_sinkhorn_iters, c.hc_eps);
    }
    launch(k_rmsnorm, dim3(1), dim3(1024), 0, st, y, y, norm, c.hidden, c.rms_eps);
}

// The cache-bound work of one layer's attention (src/model/dsv4_layer.c:224-301):
// the q heads, the KV row and the compressor step, the indexer's scores and
// top-k (or the full row list), then attention over the attended rows, for n
// activation rows whose step states are sts. A decode step: row y is
// sequence y, with its own cache. A prefill pass (pass set): row t is token t
// of sequence 0, all on one cache; each token must see the window as it
// stood at its own position, so the pass's KV rows go to staging rows (the
// ring keeps the positions before the pass), every token's row list points
// at the staging rows for positions in the pass, each token that closes a
// compressor window pools that window from the pass's projection rows and
// the compressor state as it stood before the pass, and at the end the ring
// takes the staging rows and the compressor state moves past the pass.
// Every token's arithmetic is that of its decode step.
static int attn_core(dsv4b_model *m, DevLayer &l, int n, const StepState *sts, bool pass, cudaStream_t st)
{
    const DSV4Cfg &c = m->c;
    const int hd = c.head_dim, rd = c.qk_rope, H = c.n_heads / m->world, win = c.sliding_window;
    const int ih = c.index_n_heads, id = c.index_head_dim;
    const float *cs = l.ratio ? m->cs_c : m->cs_d, *sn = l.ratio ? m->sn_c : m->sn_d;
    int rc = 0;
    // token t's compressed-row counts {avail, take}: the layer's pair (every
    // sequence of a decode step stands at the same position) or the pass's
    int *dyn = pass ? m->pdyn : l.dyn;
    const int dstride = pass ? 2 : 0, stage = pass ? l.stage_row : -1;
    // q heads, the KV row, the compressor, the indexer's q heads (or the
    // attended row list) in one launch (dsv4_layer.c:224-295)
    PrepArgs pa = {};
    pa.q = m->q;
    pa.kv = m->kv;
    pa.cache = l.kv_cache;
    pa.comp_kv = l.comp_kv;
    pa.comp_score = l.comp_score;
    pa.idx_q = m->idx_q;
    pa.kv_norm = l.kv_norm;
    pa.comp_in = m->comp_in;
    pa.comp_sc = m->comp_sc;
    pa.ape = l.ape;
    pa.cnorm = l.cnorm;
    pa.cs = cs;
    pa.sn = sn;
    pa.st = sts;
    pa.dyn = dyn;
    pa.idxs = m->idxs;
    pa.H = H;
    pa.hd = hd;
    pa.rd = rd;
    pa.win = win;
    pa.has_comp = l.has_comp;
    pa.has_idx = l.has_comp && l.has_idx;
    pa.ratio = l.ratio;
    pa.index_topk = c.index_topk;
    pa.ih = ih;
    pa.id = id;
    pa.nidx = m->nidx;
    pa.eps = c.rms_eps;
    pa.s_cache = pass ? 0 : (long)(l.kv_rows * hd);
    pa.s_comp = pass ? 0 : (long)l.comp_n;
    pa.stage = stage;
    pa.pass_nt = pass ? n : 0;
    const int blocks = H + 1 + (pa.has_comp ? 1 : 0) + (pa.has_idx ? ih : 1);
    launch(k_attn_prep, dim3(blocks, n), dim3(256), (size_t)hd * 4, st, pa);
    if (l.has_comp && l.has_idx) {
        const float scale = (1.0f / sqrtf((float)id)) * (1.0f / sqrtf((float)ih));
        // the compressed region read as contiguous rows of index_head_dim
        // floats, as the reference does (dsv4_layer.c:286-289); a pass's
        // tokens share it, in groups the head-split scratch holds
        for (int b0 = 0; b0 < n; b0 += m->ix_rows) {
            const int nb = n - b0 < m->ix_rows ? n - b0 : m->ix_rows;
            rc |= indexer_score(m->idx_scores + (size_t)b0 * m->ncomp4, m->idx_q + (size_t)b0 * ih * id,
                                l.kv_cache + (size_t)win * hd, DSV4B_DT_F32, id, pass ? 0 : (long)(l.kv_rows * hd),
                                m->idx_w + (size_t)b0 * ih, ih, id, m->ncomp4, scale, nb, st, dyn + b0 * dstride,
                                m->ix_terms, m->ix_count, dstride);
        }
        rc |= topk(m->isel, m->idx_scores, m->ncomp4, c.index_topk, n, m->ncomp4, c.index_topk, st, dyn, dstride);
        launch(k_build_idxs, dim3(n), dim3(256), 0, st, m->idxs, m->nidx, sts, win, l.has_comp, l.has_idx,
               (const int *)dyn, (const int *)m->isel, c.index_topk, dstride, stage);
    }
    // attention, each head de-rotated by the kernel that writes it
    const AttnRope rope = {cs, sn, &sts->pos, rd, pass ? (int)(sizeof(StepState) / sizeof(int)) : 0};
    rc |= sparse_attn(m->o, m->q, l.kv_cache, DSV4B_DT_F32, pass ? 0 : (long)l.kv_rows, l.sink, m->idxs, m->nidx, H,
                      hd, m->nidx, 1.0f / sqrtf((float)hd), n, m->attn_part, st, &rope);
    if (pass) launch(k_stage_commit, dim3(n + 1), dim3(256), 0, st, pa);
    return rc;
}

// One pass: enqueue only, no host synchronisation (graph-capturable).
// A decode step (rows = 0): one token of each of the nseq sequences, their
// step states at m->st. A prefill pass (rows >= 1, dsv4_layer_forward_n,
// src/model/dsv4_layer.c:856-918): rows consecutive prompt tokens of
// sequence 0, their step states at m->pst; every step runs over all rows at
// once (the cache-bound core as attn_core describes), and the head runs only
// when head is set, on the last row, advancing m->st (which then holds that
// row's position).
static int enqueue_pass(dsv4b_model *m, cudaStream_t st, int rows, bool head)
{
    const DSV4Cfg &c = m->c;
    // H: the heads of this rank (all of them on one GPU)
    const int hc = c.hc_mult, d = c.hidden, hd = c.head_dim, H = c.n_heads / m->world;
    const bool prefill = rows > 0;
    // B activation rows: a batch's sequences (every launch below covers all
    // of them: a grid dimension, or one GEMV item per row) or a pass's tokens
    const int B = prefill ? rows : m->nseq, ql = c.q_lora, ih = c.index_n_heads, id = c.index_head_dim;
    const StepState *sts = prefill ? m->pst : m->st;
    int rc = 0;
    PdlChain chain;
    float *hin = m->h, *hout = m->resid;
    Pending pend = {0, nullptr};
    const bool fused = hc_fused(c);
    m->xcall = 0;
    const Exch ex = {m->peer, m->comm, m->stepseq, m->nx, &m->xcall};
    launch(k_embed, dim3(16, B), dim3(256), 0, st, hin, m->embed, m->emb_wdt, sts, d, hc);
    for (int Li = 0; Li < c.n_layers; Li++) {
        DevLayer &l = m->L[Li];
        // ---- attention half (src/model/dsv4_layer.c:495-509), after the
        // previous FFN's post-mix; the residual stream ping-pongs between two
        // buffers, so no copy is needed
        hc_step(m, pend, hin, hout, l.hca_fn, l.hca_base, l.hca_scale, l.attn_norm, false, m->x1, st, B);
        // every projection of x1 in one launch, then both of the normalised q latent
        {
            Grp ga;
            grp_add(ga, l.wq_a, m->x1, m->qr, st, B, d, ql);
            grp_add(ga, l.wkv, m->x1, m->kv, st, B, d, hd);
            if (l.has_comp) {
                grp_add(ga, l.cwkv, m->x1, m->comp_in, st, B, d, 2 * hd);
                grp_add(ga, l.cwgate, m->x1, m->comp_sc, st, B, d, 2 * hd);
            }
            if (l.has_idx) grp_add(ga, l.iwproj, m->x1, m->idx_w, st, B, d, ih);
            rc |= grp_run(ga, st);
        }
        launch(k_rmsnorm, dim3(B), dim3(1024), 0, st, m->qr, m->qr, l.q_norm, ql, c.rms_eps);
        {
            Grp gb;
            grp_add(gb, l.wq_b, m->qr, m->q, st, B, ql, (long)H * hd);
            if (l.has_idx) grp_add(gb, l.iwq_b, m->qr, m->idx_q, st, B, ql, (long)ih * id);
            rc |= grp_run(gb, st);
        }
        // the cache-bound core, over all sequences or all of the pass's tokens
        rc |= attn_core(m, l, B, sts, prefill, st);
        // grouped low-rank output (dsv4_layer.c:303-335): the o_groups row
        // slices of wo_a, each on its own slice of o, in one launch (sharded:
        // this rank's heads are exactly its groups' slices of o)
        {
            const int gw = c.n_heads * hd / c.o_groups, gr = c.o_lora;
            const DevMat &wa = l.wo_a;
            const size_t rb = row_bytes(wa.wdt, wa.cols);
            Grp go;
            for (int g = 0; g < c.o_groups / m->world; g++) {
                DevMat sl = wa;
                sl.w = wa.w + (size_t)g * gr * rb;
                sl.s = wa.s ? wa.s + (size_t)(g * gr / wa.blk_r) * ((wa.cols + wa.blk_c - 1) / wa.blk_c) : nullptr;
                sl.rows = gr;
                sl.cols = gw;
                grp_add(go, sl, m->o + (size_t)g * gw, m->ogrp + (size_t)g * gr, st, B, (long)H * hd,
                        (long)c.o_groups * c.o_lora);
            }
            rc |= grp_run(go, st);
        }
        {
            Grp gw2;
            grp_add(gw2, l.wo_b, m->ogrp, m->blk, st, B, (long)c.o_groups * c.o_lora, d);
            rc |= grp_run(gw2, st);
        }
        // sharded: wo_b holds this rank's groups' columns, so blk is a partial
        // sum over them
        if (m->world > 1) rc |= xreduce_sum(ex, m->blk, d, st);
        // ---- FFN half: the residual is taken after attention (:511-522)
        pend = {1, nullptr};
        hc_step(m, pend, hin, hout, l.hcf_fn, l.hcf_base, l.hcf_scale, l.ffn_norm, false, m->x1, st, B);
        rc |= moe_forward(l.moe, m->ms, m->blk, m->x1, &sts->token, st, !fused, m->world > 1 ? &ex : nullptr, B,
                          m->s_ms, d, (int)(sizeof(StepState) / sizeof(int)), m->moe_perm);
        pend = {fused ? 2 : 1, &l.moe};
    }
    // a prefill pass that is not the prompt's last: only its caches matter
    if (prefill && !head) return (rc || cudaPeekAtLastError() != cudaSuccess) ? -1 : 0;
    // ---- head (src/cli/dsv4_run.c:467-474); a prefill pass reads only its
    // last token's logits (the one that picks the first generated token)
    hc_step(m, pend, hin, hout, m->hch_fn, m->hch_base, m->hch_scale, m->norm, true, m->xh, st, B);
    const int hrows = prefill ? 1 : B;
    {
        Grp gh;
        grp_add(gh, m->head, m->xh + (prefill ? (size_t)(B - 1) * d : 0), m->logits, st, hrows, d, m->head.rows);
        rc |= grp_run(gh, st);
    }
    launch(k_argmax_part, dim3(148, hrows), dim3(256), 0, st, m->am_pv, m->am_pi, m->logits, m->head.rows);
    if (m->world == 1) {
        launch(k_argmax_final, dim3(hrows), dim3(32), 0, st, m->st, m->out_tokens, m->am_pv, m->am_pi, 148, 1,
               m->prompt, m->n_prompt, (unsigned *)nullptr, m->max_pos);
    } else {
        // sharded head: each rank holds a contiguous vocabulary slice; the
        // ranks' best (value, index) pairs are gathered and reduced the same
        // way (larger value, ties to the lower index) on every rank
        launch(k_argmax_pair, dim3(1), dim3(32), 0, st, m->am_pair, m->am_pv, m->am_pi, 148,
               m->rank * m->head.rows);
        rc |= comm_allgather(m->am_pair, m->am_gather, 8, m->comm, st);
        launch(k_argmax_final, dim3(1), dim3(32), 0, st, m->st, m->out_tokens, m->am_gather,
               reinterpret_cast<const int *>(m->am_gather) + 1, m->world, 2, m->prompt, m->n_prompt, m->stepseq,
               m->max_pos);
    }
    if (cudaPeekAtLastError() != cudaSuccess) rc = -1;
    return rc ? -1 : 0;
}

static int enqueue_step(dsv4b_model *m, cudaStream_t st) { return enqueue_pass(m, st, 0, true); }

static bool build_layer_from_host(dsv4b_model *m, int Li, const DSV4LayerW &w, const DSV4ExpertW *ex)
{
    const DSV4Cfg &c = m->c;
    DevLayer &l = m->L[Li];
    bool ok = true;
    const int d = c.hidden, hd = c.head_dim, hc = c.hc_mult, mix = (2 + hc) * hc;
    l.has_comp = w.has_comp;
    l.has_idx = w.has_idx;
    if ((l.ratio != 0) != (w.has_comp != 0) || (w.has_idx && l.ratio != 4)) return false;
    l.attn_norm = up_f32(m, w.attn_norm, d, &ok);
    l.ffn_norm = up_f32(m, w.ffn_norm, d, &ok);
    l.sink = up_f32(m, w.attn.sink, c.n_heads, &ok);
    l.q_norm = up_f32(m, w.attn.q_norm, c.q_lora, &ok);
    l.kv_norm = up_f32(m, w.attn.kv_norm, hd, &ok);
    l.wq_a = up_mat(m, w.attn.wq_a, &ok);
    l.wq_b = up_mat(m, w.attn.wq_b, &ok);
    l.wkv = up_mat(m, w.attn.wkv, &ok);
    l.wo_a = up_mat(m, w.attn.wo_a, &ok);
    l.wo_b = up_mat(m, w.attn.wo_b, &ok);
    if (l.has_comp) {
        l.ape = up_f32(m, w.attn.comp.ape, (size_t)l.ratio * l.coff * hd, &ok);
        l.cnorm = up_f32(m, w.attn.comp.norm, hd, &ok);
        l.cwkv = up_mat(m, w.attn.comp.wkv, &ok);
        l.cwgate = up_mat(m, w.attn.comp.wgate, &ok);
    }
    if (l.has_idx) {
        l.iwq_b = up_mat(m, w.attn.idx.wq_b, &ok);
        l.iwproj = up_mat(m, w.attn.idx.weights_proj, &ok);
    }
    l.hca_fn = up_f32(m, w.hc_attn.fn, (size_t)mix * hc * d, &ok);
    l.hca_base = up_f32(m, w.hc_attn.base, mix, &ok);
    l.hca_scale = up_f32(m, w.hc_attn.scale, 3, &ok);
    l.hcf_fn = up_f32(m, w.hc_ffn.fn, (size_t)mix * hc * d, &ok);
    l.hcf_base = up_f32(m, w.hc_ffn.base, mix, &ok);
    l.hcf_scale = up_f32(m, w.hc_ffn.scale, 3, &ok);
    // MoE
    MoeLayer &mo = l.moe;
    mo.gate = up_mat(m, w.moe.gate, &ok);
    mo.bias = w.moe.bias ? up_f32(m, w.moe.bias, c.n_experts, &ok) : nullptr;
    mo.tid2eid = w.moe.tid2eid ? (const int64_t *)dcopy(m, w.moe.tid2eid, (size_t)c.vocab * c.topk * 8, &ok)
                               : nullptr;
    mo.fixed = nullptr;
    std::vector<const uint8_t *> tab((size_t)6 * c.n_experts);
    mo.ef16s = 1;
    for (int e = 0; e < c.n_experts && ok; e++) {
        const DSV4ExpertW &x = ex[(size_t)Li * c.n_experts + e];
        const DSV4QMat *q3[3] = { &x.w1, &x.w3, &x.w2 };
        for (int j = 0; j < 3; j++) {
            const DevMat dm = up_mat(m, *q3[j], &ok);
            tab[(size_t)(2 * j) * c.n_experts + e] = dm.w;
            tab[(size_t)(2 * j + 1) * c.n_experts + e] = dm.s;
            if (e == 0 && j == 0) { mo.efmt = dm.wdt; mo.eblk_r = dm.blk_r; mo.eblk_c = dm.blk_c; }
            mo.ef16s &= dm.f16s;
        }
    }
    const uint8_t *const *t = (const uint8_t *const *)dcopy(m, tab.data(), tab.size() * sizeof(void *), &ok);
    if (!ok) return false;
    mo.w1tab = t; mo.s1tab = t + c.n_experts;
    mo.w3tab = t + 2 * c.n_experts; mo.s3tab = t + 3 * c.n_experts;
    mo.w2tab = t + 4 * c.n_experts; mo.s2tab = t + 5 * c.n_experts;
    mo.sh[0] = up_mat(m, w.moe.shared.w1, &ok);
    mo.sh[1] = up_mat(m, w.moe.shared.w3, &ok);
    mo.sh[2] = up_mat(m, w.moe.shared.w2, &ok);
    mo.has_shared = 1;
    mo.n_experts = c.n_experts;
    mo.topk = c.topk;
    mo.hidden = d;
    mo.inter = c.moe_inter;
    mo.inter_shared = c.moe_inter * c.n_shared;
    mo.score_func = c.scoring_func == DSV4_SCORE_SIGMOID ? 2 : 1;
    mo.route_scale = c.routed_scale;
    mo.swiglu_limit = c.swiglu_limit;
    return ok;
}

}  // namespace dsv4b

using namespace dsv4b;

extern "C" void dsv4_cuda_model_free(dsv4b_model *m)
{
    if (!m) return;
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->graphed) {
        cudaGraphExecDestroy(m->exec);
        cudaGraphDestroy(m->graph);
    }
    for (auto &p : m->pgraphs) {
        cudaGraphExecDestroy(p.exec);
        cudaGraphDestroy(p.graph);
    }
    peer_close(m->peer);                 // after the graph that holds its exchanges
    comm_close(m->comm);
    for (void *p : m->allocs) cudaFree(p);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

static dsv4b_model *model_new(const DSV4Cfg *c, int max_pos, int nseq = 1)
{
    if (dsv4_cuda_init() != 0 || !c || c->n_layers < 1 || c->n_layers > DSV4_MAX_LAYERS || max_pos < 1 ||
        c->hc_mult > DSV4B_MAX_HC || c->topk > kMoeMaxTopk || c->n_experts > kMoeMaxExperts || c->n_heads > 64 ||
        c->index_topk > kTopkMaxK || nseq < 1 || nseq > DSV4B_MAX_SEQ || (nseq > 1 && !hc_fused(*c)))
        return nullptr;
    dsv4b_model *m = new dsv4b_model();
    m->c = *c;
    m->rank = 0;
    m->world = 1;
    m->nseq = nseq;
    // a one-sequence model keeps rows for a prefill pass (batched mHC needs
    // the fused form)
    m->cap = nseq > 1 ? nseq : (hc_fused(*c) ? DSV4B_MAX_PREFILL : 1);
    for (int L = 0; L < c->n_layers; L++) m->ratios[L] = c->compress_ratios ? c->compress_ratios[L] : 0;
    m->c.compress_ratios = m->ratios;
    m->max_pos = max_pos;
    m->L.resize(c->n_layers);
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess || !alloc_common(m)) {
        dsv4_cuda_model_free(m);
        return nullptr;
    }
    if (m->ncomp4 > kTopkMaxN) {
        dsv4_cuda_model_free(m);
        return nullptr;
    }
    return m;
}

// The kernel nodes of a captured graph, or -1.
static int graph_kernels(cudaGraph_t g)
{
    size_t n = 0;
    if (cudaGraphGetNodes(g, nullptr, &n) != cudaSuccess) return -1;
    std::vector<cudaGraphNode_t> nodes(n);
    if (n && cudaGraphGetNodes(g, nodes.data(), &n) != cudaSuccess) return -1;
    int k = 0;
    for (size_t i = 0; i < n; i++) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(nodes[i], &t) != cudaSuccess) return -1;
        k += t == cudaGraphNodeTypeKernel;
    }
    return k;
}

// One prefill pass of nt tokens (their step states already at m->pst), on
// m->stream: eagerly the first time its shape is seen, captured the second
// time, its graph replayed after that. Returns the kernels it launched (-1
// if unknown: an eager pass), or -2 on failure.
static int run_pass(dsv4b_model *m, int nt, bool last)
{
    const int key = nt * 2 + (last ? 1 : 0);
    for (auto &p : m->pgraphs)
        if (p.key == key) return cudaGraphLaunch(p.exec, m->stream) == cudaSuccess ? p.kernels : -2;
    if (std::find(m->pseen.begin(), m->pseen.end(), key) == m->pseen.end()) {
        m->pseen.push_back(key);
        return enqueue_pass(m, m->stream, nt, last) ? -2 : -1;
    }
    dsv4b_model::PassGraph p = {key, 0, nullptr, nullptr};
    if (cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return -2;
    const int rc = enqueue_pass(m, m->stream, nt, last);
    const cudaError_t e = cudaStreamEndCapture(m->stream, &p.graph);
    if (rc || e != cudaSuccess || cudaGraphInstantiate(&p.exec, p.graph, 0) != cudaSuccess) {
        if (p.graph) cudaGraphDestroy(p.graph);
        return -2;
    }
    p.kernels = graph_kernels(p.graph);
    m->pgraphs.push_back(p);
    return cudaGraphLaunch(p.exec, m->stream) == cudaSuccess ? p.kernels : -2;
}

extern "C" dsv4b_model *dsv4_cuda_model_create_batch(const DSV4Cfg *c, const DSV4ModelW *mw,
                                                     const DSV4LayerW *layers, const DSV4ExpertW *experts,
                                                     int max_pos, int n_seq)
{
    if (!mw || !layers || !experts) return nullptr;
    dsv4b_model *m = model_new(c, max_pos, n_seq);
    if (!m) return nullptr;
    bool ok = true;
    for (int L = 0; L < c->n_layers && ok; L++) ok = build_layer_from_host(m, L, layers[L], experts);
    const int d = c->hidden, hc = c->hc_mult;
    m->emb_wdt = mw->wdt;
    m->embed = dcopy(m, mw->embed, (size_t)c->vocab * d * (mw->wdt == DSV4_WBF16 ? 2 : 4), &ok);
    DSV4QMat hq = { mw->head, nullptr, mw->wdt, c->vocab, d, 0, 0 };
    m->head = up_mat(m, hq, &ok);
    m->norm = up_f32(m, mw->norm, d, &ok);
    m->hch_fn = up_f32(m, mw->hc_head.fn, (size_t)hc * hc * d, &ok);
    m->hch_base = up_f32(m, mw->hc_head.base, hc, &ok);
    m->hch_scale = up_f32(m, mw->hc_head.scale, 1, &ok);
    if (!ok || cudaDeviceSynchronize() != cudaSuccess) {
        dsv4_cuda_model_free(m);
        return nullptr;
    }
    return m;
}

extern "C" dsv4b_model *dsv4_cuda_model_create(const DSV4Cfg *c, const DSV4ModelW *mw, const DSV4LayerW *layers,
                                               const DSV4ExpertW *experts, int max_pos)
{
    return dsv4_cuda_model_create_batch(c, mw, layers, experts, max_pos, 1);
}

extern "C" int dsv4b_model_n_seq(const dsv4b_model *m) { return m ? m->nseq : -1; }

extern "C" int dsv4b_model_begin_batch(dsv4b_model *m, const int *prompts, int n_prompt)
{
    if (!m || !prompts || n_prompt < 1 || n_prompt > m->max_pos) return -1;
    const int B = m->nseq;
    for (int i = 0; i < B * n_prompt; i++)
        if (prompts[i] < 0 || prompts[i] >= m->c.vocab) return -1;
    m->n_prompt = n_prompt;
    // sequence b's prompt at row b of the max_pos-wide prompt table
    for (int b = 0; b < B; b++)
        DSV4B_CUDA_OK(cudaMemcpyAsync(m->prompt + (size_t)b * m->max_pos, prompts + (size_t)b * n_prompt,
                                      (size_t)n_prompt * 4, cudaMemcpyHostToDevice, m->stream));
    std::vector<StepState> s0v(B);
    for (int b = 0; b < B; b++) s0v[b] = { prompts[(size_t)b * n_prompt], 0 };
    const StepState *s0 = s0v.data();
    const size_t s0b = (size_t)B * sizeof(StepState);
    if (reset_state(m)) return -1;
    DSV4B_CUDA_OK(cudaMemcpyAsync(m->st, s0, s0b, cudaMemcpyHostToDevice, m->stream));
    if (!m->graphed) {
        // one eager step sets every kernel attribute, then the state is reset
        // and the step is captured once for all positions
        if (enqueue_step(m, m->stream)) return -1;
        DSV4B_CUDA_OK(cudaStreamSynchronize(m->stream));
        if (reset_state(m)) return -1;
        DSV4B_CUDA_OK(cudaMemcpyAsync(m->st, s0, s0b, cudaMemcpyHostToDevice, m->stream));
        DSV4B_CUDA_OK(cudaStreamSynchronize(m->stream));
        DSV4B_CUDA_OK(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
        const int rc = enqueue_step(m, m->stream);
        cudaGraph_t g = nullptr;
        const cudaError_t e = cudaStreamEndCapture(m->stream, &g);
        if (rc || e != cudaSuccess) return -1;
        DSV4B_CUDA_OK(cudaGraphInstantiate(&m->exec, g, 0));
        m->graph = g;
        m->graphed = 1;
    }
    DSV4B_CUDA_OK(cudaStreamSynchronize(m->stream));
    return 0;
}

extern "C" int dsv4_cuda_model_begin(dsv4b_model *m, const int *prompt, int n_prompt)
{
    if (!m || m->nseq != 1) return -1;
    return dsv4b_model_begin_batch(m, prompt, n_prompt);
}

extern "C" int dsv4b_model_step_async(dsv4b_model *m, void *stream)
{
    if (!m || !m->graphed) return -1;
    DSV4B_CUDA_OK(cudaGraphLaunch(m->exec, stream ? (cudaStream_t)stream : m->stream));
    return 0;
}

extern "C" int dsv4_cuda_model_step(dsv4b_model *m, int *token, float *logits)
{
    if (!m || !m->graphed || m->nseq != 1) return -1;
    StepState s;
    DSV4B_CUDA_OK(cudaMemcpyAsync(&s, m->st, sizeof s, cudaMemcpyDeviceToHost, m->stream));
    DSV4B_CUDA_OK(cudaStreamSynchronize(m->stream));
    if (s.pos >= m->max_pos) return -1;
    DSV4B_CUDA_OK(cudaGraphLaunch(m->exec, m->stream));
    if (token) DSV4B_CUDA_OK(cudaMemcpyAsync(token, m->out_tokens + s.pos, 4, cudaMemcpyDeviceToHost, m->stream));
    if (logits)
        DSV4B_CUDA_OK(cudaMemcpyAsync(logits, m->logits, (size_t)m->c.vocab * 4, cudaMemcpyDeviceToHost, m->stream));
    DSV4B_CUDA_OK(cudaStreamSynchronize(m->stream));
    return 0;
}

extern "C" int dsv4b_model_generate_batch(dsv4b_model *m, const int *prompts, int n_prompt, int n_gen, int *out)
{
    if (dsv4b_model_begin_batch(m, prompts, n_prompt) != 0) return -1;
    const int steps = n_prompt + n_gen;
    if (steps > m->max_pos) return -1;
    for (int i = 0; i < steps; i++) DSV4B_CUDA_OK(cudaGraphLaunch(m->exec, m->stream));
    // position p emits the token after it; the generated ones start at n_prompt-1
    for (int b = 0; b < m->nseq; b++)
        DSV4B_CUDA_OK(cudaMemcpyAsync(out + (size_t)b * (n_gen + 1),
                                      m->out_tokens + (size_t)b * m->max_pos + n_prompt - 1, (size_t)(n_gen + 1) * 4,
                                      cudaMemcpyDeviceToHost, m->stream));
    DSV4B_CUDA_OK(cudaStreamSynchronize(m->stream));
    return n_gen + 1;
}

extern "C" int dsv4_cuda_model_generate(dsv4b_model *m, const int *prompt, int n_prompt, int n_gen, int *out)
{
    if (!m || m->nseq != 1) return -1;
    return dsv4b_model_generate_batch(m, prompt, n_prompt, n_gen, out);
}

extern "C" int dsv4b_model_prefill(dsv4b_model *m, const int *prompt, int n_prompt, int chunk)
{
    if (!m || m->nseq != 1 || m->world != 1 || chunk < 1 || chunk > m->cap || !dsv4b::hc_fused(m->c)) return -1;
    if (dsv4b_model_begin_batch(m, prompt, n_prompt) != 0) return -1;
    // every prompt token's step state; pass p0 copies its slice
    std::vector<dsv4b::StepState> s(n_prompt);
    for (int i = 0; i < n_prompt; i++) s[i] = { prompt[i], i };
    int kernels = 0;
    for (int p0 = 0; p0 < n_prompt; p0 += chunk) {
        const int nt = std::min(chunk, n_prompt - p0);
        const bool last = p0 + nt >= n_prompt;
        DSV4B_CUDA_OK(cudaMemcpyAsync(m->pst, s.data() + p0, (size_t)nt * sizeof(dsv4b::StepState),
                                      cudaMemcpyHostToDevice, m->stream));
        // the head of the last pass advances the decode state from the last
        // prompt position, as a per-token run's last prompt step does
        if (last)
            DSV4B_CUDA_OK(cudaMemcpyAsync(m->st, s.data() + n_prompt - 1, sizeof(dsv4b::StepState),
                                          cudaMemcpyHostToDevice, m->stream));
        const int k = run_pass(m, nt, last);
        if (k == -2) return -1;
        kernels = (kernels < 0 || k < 0) ? -1 : kernels + k;
    }
    m->pf_kernels = kernels;
    int tok = -1;
    DSV4B_CUDA_OK(cudaMemcpyAsync(&tok, m->out_tokens + n_prompt - 1, 4, cudaMemcpyDeviceToHost, m->stream));
    DSV4B_CUDA_OK(cudaStreamSynchronize(m->stream));
    return tok;
}

extern "C" int dsv4b_model_generate_prefill(dsv4b_model *m, const int *prompt, int n_prompt, int n_gen, int chunk,
                                            int *out)
{
    if (!m || !prompt || !out || n_prompt < 1 || n_gen < 0 || n_prompt + n_gen > m->max_pos) return -1;
    if (dsv4b_model_prefill(m, prompt, n_prompt, chunk) < 0) return -1;
    for (int i = 0; i < n_gen; i++) DSV4B_CUDA_OK(cudaGraphLaunch(m->exec, m->stream));
    DSV4B_CUDA_OK(cudaMemcpyAsync(out, m->out_tokens + n_prompt - 1, (size_t)(n_gen + 1) * 4, cudaMemcpyDeviceToHost,
                                  m->stream));
    DSV4B_CUDA_OK(cudaStreamSynchronize(m->stream));
    return n_gen + 1;
}

// ------------------------------------------------------- synthetic models

namespace dsv4b {

struct Synth {
    dsv4b_model *m;
    uint64_t seed, tensor = 0;
    int rank = 0, world = 1;
    bool ok = true;
    uint64_t next_key() { return (seed * 0x9E3779B97F4A7C15ull) ^ (++tensor * 0xD1B54A32D192ED03ull); }
    void launched()
    {
        if (cudaPeekAtLastError() != cudaSuccess) ok = false;
    }
    // the [nrows][ncols] slice at element base (row stride gstride) of the
    // next tensor; a whole tensor is the slice at 0 of itself
    void *slice(size_t bytes, int nrows, int ncols, int kind, float a, float b, size_t base, size_t gstride)
    {
        const uint64_t key = next_key();
        if (!ok) return nullptr;
        void *p = dalloc(m, bytes);
        if (!p) { ok = false; return nullptr; }
        k_synth_slice<<<1184, 256, 0, m->stream>>>(p, nrows, ncols, kind, a, b, key, base, gstride);
        launched();
        return p;
    }
    float *f32n(size_t n, float a, float b) { return (float *)slice(n * 4, 1, (int)n, 0, a, b, 0, n); }
    float *f32u(size_t n, float a, float b) { return (float *)slice(n * 4, 1, (int)n, 1, a, b, 0, n); }
    float *f32n_part(size_t n, size_t off, size_t cnt, float a, float b)
    {
        return (float *)slice(cnt * 4, 1, (int)cnt, 0, a, b, off, n);
    }
    // FP8 128x128, codes of N(0, 0.02) at scale 2^-10: rows [r0, r0 + nr) and
    // columns [c0, c0 + nc) of a rows x cols matrix (128-aligned slices)
    DevMat fp8(int rows, int cols, int r0 = 0, int nr = -1, int c0 = 0, int nc = -1)
    {
        if (nr < 0) nr = rows;
        if (nc < 0) nc = cols;
        DevMat d = {nullptr, nullptr, DSV4_WFP8, nr, nc, 128, 128};
        const size_t sb = (size_t)((nr + 127) / 128) * ((nc + 127) / 128);
        d.w = (const uint8_t *)slice((size_t)nr * nc, nr, nc, 3, 0.f, 0.02f / 0.0009765625f,
                                     (size_t)r0 * cols + c0, cols);
        d.s = (const uint8_t *)slice(sb, 1, (int)sb, 5, 117.f, 0.f, 0, sb);      // 2^-10
        return d;
    }
    DevMat bf16(int rows, int cols, float sigma, int r0 = 0, int nr = -1)
    {
        if (nr < 0) nr = rows;
        DevMat d = {nullptr, nullptr, DSV4_WBF16, nr, cols, 0, 0};
        d.w = (const uint8_t *)slice((size_t)nr * cols * 2, nr, cols, 2, 0.f, sigma, (size_t)r0 * cols, cols);
        return d;
    }
};

static bool synth_layer(Synth &S, int Li)
{
    dsv4b_model *m = S.m;
    const DSV4Cfg &c = m->c;
    DevLayer &l = m->L[Li];
    const int d = c.hidden, hd = c.head_dim, hc = c.hc_mult, mix = (2 + hc) * hc, H = c.n_heads;
    // this rank's share: heads (and so o_groups), the wo_b columns of those
    // groups, every expert's inter slice
    int sp[2 * DSV4B_SHARD_NDIM];
    if (dsv4b_shard_plan(&c, S.world, S.rank, sp) < 0) return false;
    const int *hs = sp + 2 * DSV4B_SHARD_HEADS, *qs = sp + 2 * DSV4B_SHARD_QROWS, *os = sp + 2 * DSV4B_SHARD_OLORA;
    l.has_comp = l.ratio != 0;
    l.has_idx = l.ratio == 4;
    l.attn_norm = S.f32n(d, 1.f, 0.1f);
    l.ffn_norm = S.f32n(d, 1.f, 0.1f);
    l.sink = S.f32n_part(H, (size_t)hs[0], hs[1], 0.f, 1.f);
    l.q_norm = S.f32n(c.q_lora, 1.f, 0.1f);
    l.kv_norm = S.f32n(hd, 1.f, 0.1f);
    l.wq_a = S.fp8(c.q_lora, d);
    l.wq_b = S.fp8(H * hd, c.q_lora, qs[0], qs[1]);
    l.wkv = S.fp8(hd, d);
    l.wo_a = S.fp8(c.o_groups * c.o_lora, H * hd / c.o_groups, os[0], os[1]);
    l.wo_b = S.fp8(d, c.o_groups * c.o_lora, 0, d, os[0], os[1]);
    if (l.has_comp) {
        l.ape = S.f32n((size_t)l.ratio * l.coff * hd, 0.f, 0.1f);
        l.cnorm = S.f32n(hd, 1.f, 0.1f);
        l.cwkv = S.bf16(l.coff * hd, d, 0.02f);
        l.cwgate = S.bf16(l.coff * hd, d, 0.02f);
    }
    if (l.has_idx) {
        l.iwq_b = S.fp8(c.index_n_heads * c.index_head_dim, c.q_lora);
        l.iwproj = S.bf16(c.index_n_heads, d, 0.02f);
    }
    l.hca_fn = S.f32n((size_t)mix * hc * d, 0.f, 0.02f);
    l.hca_base = S.f32n(mix, 0.f, 0.5f);
    l.hca_scale = S.f32u(3, 0.5f, 0.5f);
    l.hcf_fn = S.f32n((size_t)mix * hc * d, 0.f, 0.02f);
    l.hcf_base = S.f32n(mix, 0.f, 0.5f);
    l.hcf_scale = S.f32u(3, 0.5f, 0.5f);
    MoeLayer &mo = l.moe;
    mo.gate = S.bf16(c.n_experts, d, 0.02f);
    mo.fixed = nullptr;
    if (Li < c.num_hash_layers) {
        int64_t *t = (int64_t *)dalloc(m, (size_t)c.vocab * c.topk * 8);
        if (!t) return false;
        k_synth_tid2eid<<<256, 256, 0, m->stream>>>(t, c.vocab, c.topk, c.n_experts, S.seed + 77 * Li);
        mo.tid2eid = t;
        mo.bias = nullptr;
    } else {
        mo.tid2eid = nullptr;
        mo.bias = S.f32n(c.n_experts, 0.f, 0.05f);
    }
    // routed experts: one stream of codes per layer (every expert's w1, w3,
    // w2), then the scales; this rank keeps its inter slice of each expert
    const size_t I = sp[2 * DSV4B_SHARD_INTER + 1], E = c.n_experts;
    const size_t cw = I * d / 2, cper = 3 * cw, sw = I * d / 32, sper = 3 * sw;
    uint8_t *codes = (uint8_t *)dalloc(m, E * cper), *scales = (uint8_t *)dalloc(m, E * sper);
    if (!codes || !scales) return false;
    const uint64_t ckey = S.next_key();
    k_synth_experts<<<1184, 256, 0, m->stream>>>(codes, (int)E, d, c.moe_inter, sp[2 * DSV4B_SHARD_INTER], (int)I, 0.02f / 0.015625f,
                                                   ckey);                    // e2m1 of N(0,0.02) / 2^-6
    S.launched();
    S.next_key();
    k_synth_slice<<<1184, 256, 0, m->stream>>>(scales, 1, (int)(E * sper), 5, 121.f, 0.f, 0, 0, E * sper);
    S.launched();                                                            // 2^-6
    std::vector<const uint8_t *> tab(6 * E);
    for (size_t e = 0; e < E; e++) {
        for (int j = 0; j < 3; j++) {
            tab[(2 * j) * E + e] = codes + e * cper + j * cw;
            tab[(2 * j + 1) * E + e] = scales + e * sper + j * sw;
        }
    }
    bool ok = true;
    const uint8_t *const *t = (const uint8_t *const *)dcopy(m, tab.data(), tab.size() * sizeof(void *), &ok);
    if (!ok) return false;
    mo.w1tab = t; mo.s1tab = t + E;
    mo.w3tab = t + 2 * E; mo.s3tab = t + 3 * E;
    mo.w2tab = t + 4 * E; mo.s2tab = t + 5 * E;
    mo.efmt = DSV4_WFP4; mo.eblk_r = 1; mo.eblk_c = 32;
    mo.ef16s = 1;                                               // every scale is 2^-6
    const int Is = c.moe_inter * c.n_shared, Is0 = sp[2 * DSV4B_SHARD_SHARED_INTER], Isl = sp[2 * DSV4B_SHARD_SHARED_INTER + 1];
    mo.sh[0] = S.fp8(Is, d, Is0, Isl);
    mo.sh[1] = S.fp8(Is, d, Is0, Isl);
    mo.sh[2] = S.fp8(d, Is, 0, d, Is0, Isl);
    mo.has_shared = 1;
    mo.n_experts = c.n_experts;
    mo.topk = c.topk;
    mo.hidden = d;
    mo.inter = (int)I;
    mo.inter_shared = Isl;
    mo.score_func = c.scoring_func == DSV4_SCORE_SIGMOID ? 2 : 1;
    mo.route_scale = c.routed_scale;
    mo.swiglu_limit = c.swiglu_limit;
    return S.ok;
}

}  // namespace dsv4b

// Whether a model of this configuration splits over `world` GPUs: heads and
// o_groups by rank (a rank's heads are its groups' slices of o), wo_a / wo_b
// slices on 128-row / -column FP8 blocks, every expert's inter slice a whole
// number of 32-column FP4 scale blocks, the shared expert's on 128 blocks,
// and the vocabulary.
extern "C" int dsv4b_shard_check(const DSV4Cfg *c, int world)
{
    if (!c || world < 1 || world > 64) return -1;
    if (world == 1) return 0;
    const int ogl = c->o_groups / world, orl = ogl * c->o_lora, Hl = c->n_heads / world;
    const int il = c->moe_inter / world, isl = c->moe_inter * c->n_shared / world;
    const bool ok = c->n_heads % world == 0 && c->o_groups % world == 0 && c->n_heads % c->o_groups == 0 &&
                    (Hl * c->head_dim) % 128 == 0 && orl % 128 == 0 && c->moe_inter % world == 0 && il % 32 == 0 &&
                    (c->moe_inter * c->n_shared) % world == 0 && isl % 128 == 0 && c->vocab % world == 0 &&
                    c->n_shared >= 1;
    return ok ? 0 : -1;
}

extern "C" int dsv4b_shard_plan(const DSV4Cfg *c, int world, int rank, int *out)
{
    if (!out || dsv4b_shard_check(c, world) != 0 || rank < 0 || rank >= world) return -1;
    const int G = world, r = rank, Hl = c->n_heads / G, ogl = c->o_groups / G, orl = ogl * c->o_lora;
    const int il = c->moe_inter / G, isl = c->moe_inter * c->n_shared / G, vl = c->vocab / G;
    const int share[DSV4B_SHARD_NDIM] = { Hl, Hl * c->head_dim, ogl, orl, il, isl, vl };
    for (int k = 0; k < DSV4B_SHARD_NDIM; k++) {
        out[2 * k] = r * share[k];
        out[2 * k + 1] = share[k];
    }
    return DSV4B_SHARD_NDIM;
}

extern "C" size_t dsv4b_nccl_id_bytes(void) { return comm_id_bytes(); }

// 0 while every exchange of a sharded model has completed in time; 1 once a
// peer exchange gave up waiting for a rank (its results are then invalid).
extern "C" int dsv4b_model_comm_status(const dsv4b_model *m) { return m ? peer_status(m->peer) : -1; }

extern "C" int dsv4b_nccl_unique_id(void *out) { return comm_unique_id(out); }

// A synthetic model, or this rank's share of one: the tensors of rank r are
// exactly the corresponding slices of the single-GPU model of the same seed.
static dsv4b_model *synthetic_create(const DSV4Cfg *c, int max_pos, unsigned long long seed, int rank, int world,
                                     const void *nccl_id, int nseq)
{
    if (!c || dsv4b_shard_check(c, world) != 0 || rank < 0 || rank >= world || (world > 1 && !nccl_id) ||
        (world > 1 && nseq != 1)) {
        fprintf(stderr, "dsv4_b200: configuration does not split over %d GPUs (or bad rank %d)\n", world, rank);
        return nullptr;
    }
    dsv4b_model *m = model_new(c, max_pos, nseq);
    if (!m) return nullptr;
    m->rank = rank;
    m->world = world;
    if (comm_open(&m->comm, rank, world, nccl_id) != 0) {
        dsv4_cuda_model_free(m);
        return nullptr;
    }
    // the one-shot peer exchange unless DSV4B_PEER=0 (then NCCL all-reduces)
    const char *pe = getenv("DSV4B_PEER");
    if (world > 1 && !(pe && pe[0] == '0'))
        peer_open(&m->peer, rank, world, (c->topk + 1) * c->hidden, m->comm, m->stream);
    dsv4b::Synth S;
    S.m = m;
    S.seed = seed;
    S.rank = rank;
    S.world = world;
    bool ok = true;
    for (int L = 0; L < c->n_layers && ok; L++) ok = dsv4b::synth_layer(S, L);
    const int d = c->hidden, hc = c->hc_mult;
    int sp[2 * DSV4B_SHARD_NDIM];
    dsv4b_shard_plan(c, world, rank, sp);
    const int *vs = sp + 2 * DSV4B_SHARD_VOCAB;
    if (ok) {
        m->emb_wdt = DSV4_WBF16;
        m->embed = S.bf16(c->vocab, d, 1.0f).w;
        m->head = S.bf16(c->vocab, d, 0.02f, vs[0], vs[1]);
        m->norm = S.f32n(d, 1.f, 0.1f);
        m->hch_fn = S.f32n((size_t)hc * hc * d, 0.f, 0.02f);
        m->hch_base = S.f32n(hc, 0.f, 0.5f);
        m->hch_scale = S.f32u(1, 0.5f, 0.5f);
        ok = S.ok;
    }
    if (!ok || cudaStreamSynchronize(m->stream) != cudaSuccess) {
        fprintf(stderr, "dsv4_b200: synthetic model did not fit or failed (%s)\n",
                cudaGetErrorString(cudaGetLastError()));
        dsv4_cuda_model_free(m);
        return nullptr;
    }
    return m;
}

extern "C" dsv4b_model *dsv4_cuda_model_create_synthetic_sharded(const DSV4Cfg *c, int max_pos,
                                                                unsigned long long seed, int rank, int world,
                                                                const void *nccl_id)
{
    return synthetic_create(c, max_pos, seed, rank, world, nccl_id, 1);
}

extern "C" dsv4b_model *dsv4_cuda_model_create_synthetic(const DSV4Cfg *c, int max_pos, unsigned long long seed)
{
    return synthetic_create(c, max_pos, seed, 0, 1, nullptr, 1);
}

extern "C" dsv4b_model *dsv4_cuda_model_create_synthetic_batch(const DSV4Cfg *c, int max_pos,
                                                              unsigned long long seed, int n_seq)
{
    return synthetic_create(c, max_pos, seed, 0, 1, nullptr, n_seq);
}

extern "C" int dsv4_cuda_model_decode(dsv4b_model *m, int token, int pos, int *next_token)
{
    if (!m || !m->graphed || m->nseq != 1 || pos < 0 || pos >= m->max_pos || token < 0 || token >= m->c.vocab) return -1;
    const dsv4b::StepState s = { token, pos };
    DSV4B_CUDA_OK(cudaMemcpyAsync(m->st, &s, sizeof s, cudaMemcpyHostToDevice, m->stream));
    DSV4B_CUDA_OK(cudaGraphLaunch(m->exec, m->stream));
    DSV4B_CUDA_OK(cudaMemcpyAsync(next_token, m->out_tokens + pos, 4, cudaMemcpyDeviceToHost, m->stream));
    DSV4B_CUDA_OK(cudaStreamSynchronize(m->stream));
    return 0;
}

extern "C" int dsv4b_model_decode_batch(dsv4b_model *m, const int *tokens, int pos, int *next_tokens)
{
    if (!m || !m->graphed || !tokens || !next_tokens || pos < 0 || pos >= m->max_pos) return -1;
    const int B = m->nseq;
    std::vector<dsv4b::StepState> s(B);
    for (int b = 0; b < B; b++) {
        if (tokens[b] < 0 || tokens[b] >= m->c.vocab) return -1;
        s[b] = { tokens[b], pos };
    }
    DSV4B_CUDA_OK(cudaMemcpyAsync(m->st, s.data(), (size_t)B * sizeof(dsv4b::StepState), cudaMemcpyHostToDevice,
                                  m->stream));
    DSV4B_CUDA_OK(cudaGraphLaunch(m->exec, m->stream));
    // token b at out_tokens[b][pos]: one strided copy
    DSV4B_CUDA_OK(cudaMemcpy2DAsync(next_tokens, 4, m->out_tokens + pos, (size_t)m->max_pos * 4, 4, B,
                                    cudaMemcpyDeviceToHost, m->stream));
    DSV4B_CUDA_OK(cudaStreamSynchronize(m->stream));
    return 0;
}

extern "C" int dsv4_cuda_model_step_kernels(const dsv4b_model *m)
{
    if (!m || !m->graphed) return -1;
    return graph_kernels(m->graph);
}

extern "C" int dsv4b_model_prefill_kernels(const dsv4b_model *m) { return m ? m->pf_kernels : -1; }

extern "C" void *dsv4b_model_stream(const dsv4b_model *m) { return m ? (void *)m->stream : nullptr; }

extern "C" size_t dsv4_cuda_model_bytes(const dsv4b_model *m)
{
    size_t b = 0;
    (void)m;
    size_t fr = 0, tot = 0;
    if (cudaMemGetInfo(&fr, &tot) == cudaSuccess) b = tot - fr;
    return b;
}

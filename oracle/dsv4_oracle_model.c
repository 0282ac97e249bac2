/* dsv4_oracle_model.c - CPU restatement of one whole decode token.
 *
 * TEST INFRASTRUCTURE ONLY (see dsv4_oracle.h). Restates, over the
 * reference's own weight structs (include/dsv4_types.h mirrors
 * include/dsv4/dsv4.h):
 *   dsv4_layer_forward   src/model/dsv4_layer.c:487-523
 *   attention()          src/model/dsv4_layer.c:213-336
 *   moe()                src/model/dsv4_layer.c:369-484
 *   dsv4_state_init      src/model/dsv4_layer.c:80-108
 *   the token loop, hc_head and argmax of src/cli/dsv4_run.c:94-116,444-483
 * using the kernel restatements of dsv4_oracle.c, which are bit-identical to
 * the reference's C. Experts come from an array [n_layers][n_experts] instead
 * of the reference's streaming cache; the arithmetic does not depend on where
 * an expert's bytes come from.
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "dsv4_oracle.h"
#include "../include/dsv4_types.h"

typedef struct {
    float *kv_cache, *comp_kv, *comp_score;
    int n_compressed;
} LState;

typedef struct dsv4o_model {
    DSV4Cfg c;
    int ratios[DSV4_MAX_LAYERS];
    const DSV4ModelW *mw;
    const DSV4LayerW *lw;
    const DSV4ExpertW *ex;
    int max_pos;
    LState *st;
    float *cs_d, *sn_d, *cs_c, *sn_c;
    /* scratch */
    float *h, *x1, *resid, *post, *comb, *mixes, *qr, *q, *kv, *o, *ogrp, *blk;
    float *comp_in, *comp_sc, *idx_q, *idx_w, *idx_scores, *attn_scratch;
    float *gate_scores, *gate_orig, *eg, *eu, *eh, *acc, *xh, *logits;
    int *idxs;
} dsv4o_model;

static void mmq(float *y, const float *x, const DSV4QMat *m) { dsv4o_mmq(y, x, (const dsv4o_mat *)m); }

static void *xalloc(size_t n)
{
    void *p = calloc(n ? n : 1, 1);
    if (!p) { fprintf(stderr, "dsv4_oracle_model: out of memory\n"); abort(); }
    return p;
}

dsv4o_model *dsv4o_model_create(const void *cfg, const void *mwv, const void *lwv, const void *exv,
                                int max_pos)
{
    const DSV4Cfg *c = (const DSV4Cfg *)cfg;
    const DSV4ModelW *mw = (const DSV4ModelW *)mwv;
    const DSV4LayerW *lw = (const DSV4LayerW *)lwv;
    const DSV4ExpertW *ex = (const DSV4ExpertW *)exv;
    dsv4o_model *m = (dsv4o_model *)xalloc(sizeof *m);
    m->c = *c;
    for (int L = 0; L < c->n_layers && L < DSV4_MAX_LAYERS; L++) m->ratios[L] = c->compress_ratios[L];
    m->c.compress_ratios = m->ratios;
    m->mw = mw; m->lw = lw; m->ex = ex; m->max_pos = max_pos;
    const int hd = c->head_dim, hc = c->hc_mult, d = c->hidden, win = c->sliding_window;
    m->st = (LState *)xalloc(sizeof(LState) * c->n_layers);
    for (int L = 0; L < c->n_layers; L++) {
        const int ratio = m->ratios[L] > 0 ? m->ratios[L] : 0, coff = ratio == 4 ? 2 : 1;
        const size_t ncomp = ratio ? (size_t)(max_pos / ratio + 1) : 0;
        m->st[L].kv_cache = (float *)xalloc(((size_t)win + ncomp) * hd * 4);
        if (ratio) {
            const size_t cn = (size_t)coff * ratio * coff * hd;
            m->st[L].comp_kv = (float *)xalloc(cn * 4);
            m->st[L].comp_score = (float *)xalloc(cn * 4);
            for (size_t i = 0; i < cn; i++) m->st[L].comp_score[i] = -INFINITY;
        }
    }
    const int half = c->qk_rope / 2;
    m->cs_d = (float *)xalloc((size_t)max_pos * half * 4); m->sn_d = (float *)xalloc((size_t)max_pos * half * 4);
    m->cs_c = (float *)xalloc((size_t)max_pos * half * 4); m->sn_c = (float *)xalloc((size_t)max_pos * half * 4);
    dsv4o_rope_table(m->cs_d, m->sn_d, c->qk_rope, max_pos, 0, c->rope_theta, c->yarn_factor,
                     c->yarn_beta_fast, c->yarn_beta_slow);
    dsv4o_rope_table(m->cs_c, m->sn_c, c->qk_rope, max_pos, c->yarn_orig_ctx, c->compress_rope_theta,
                     c->yarn_factor, c->yarn_beta_fast, c->yarn_beta_slow);
    const size_t big = (size_t)(d > c->q_lora ? d : c->q_lora);
    const int nidx = win + c->index_topk;
    const int inter = c->moe_inter * (c->n_shared > 1 ? c->n_shared : 1);
    m->h = (float *)xalloc((size_t)hc * d * 4);
    m->x1 = (float *)xalloc((size_t)d * 4);
    m->resid = (float *)xalloc((size_t)hc * d * 4);
    m->post = (float *)xalloc(64); m->comb = (float *)xalloc(256); m->mixes = (float *)xalloc(512);
    m->qr = (float *)xalloc(big * 4);
    m->q = (float *)xalloc((size_t)c->n_heads * hd * 4);
    m->kv = (float *)xalloc((size_t)hd * 4);
    m->o = (float *)xalloc((size_t)c->n_heads * hd * 4);
    m->ogrp = (float *)xalloc((size_t)c->o_groups * c->o_lora * 4);
    m->blk = (float *)xalloc((size_t)d * 4);
    m->comp_in = (float *)xalloc((size_t)2 * hd * 4); m->comp_sc = (float *)xalloc((size_t)2 * hd * 4);
    m->idx_q = (float *)xalloc((size_t)c->index_n_heads * c->index_head_dim * 4);
    m->idx_w = (float *)xalloc((size_t)c->index_n_heads * 4);
    m->idx_scores = (float *)xalloc((size_t)(max_pos + 1) * 4);
    m->attn_scratch = (float *)xalloc((size_t)c->n_heads * nidx * 4);
    m->idxs = (int *)xalloc((size_t)nidx * 4);
    m->gate_scores = (float *)xalloc((size_t)c->n_experts * 4);
    m->gate_orig = (float *)xalloc((size_t)c->n_experts * 4);
    m->eg = (float *)xalloc((size_t)inter * 4); m->eu = (float *)xalloc((size_t)inter * 4);
    m->eh = (float *)xalloc((size_t)inter * 4);
    m->acc = (float *)xalloc((size_t)(c->topk + 1) * d * 4);
    m->xh = (float *)xalloc((size_t)d * 4);
    m->logits = (float *)xalloc((size_t)c->vocab * 4);
    return m;
}

void dsv4o_model_free(dsv4o_model *m)
{
    if (!m) return;
    for (int L = 0; L < m->c.n_layers; L++) {
        free(m->st[L].kv_cache); free(m->st[L].comp_kv); free(m->st[L].comp_score);
    }
    free(m->st);
    free(m->cs_d); free(m->sn_d); free(m->cs_c); free(m->sn_c);
    free(m->h); free(m->x1); free(m->resid); free(m->post); free(m->comb); free(m->mixes);
    free(m->qr); free(m->q); free(m->kv); free(m->o); free(m->ogrp); free(m->blk);
    free(m->comp_in); free(m->comp_sc); free(m->idx_q); free(m->idx_w); free(m->idx_scores);
    free(m->attn_scratch); free(m->idxs); free(m->gate_scores); free(m->gate_orig);
    free(m->eg); free(m->eu); free(m->eh); free(m->acc); free(m->xh); free(m->logits);
    free(m);
}

/* src/model/dsv4_layer.c:213-336 */
static void attention(dsv4o_model *m, float *out, const float *x, const DSV4LayerW *w, LState *st,
                      const float *cs, const float *sn, int pos, int n_idx)
{
    const DSV4Cfg *c = &m->c;
    const int hd = c->head_dim, rd = c->qk_rope, H = c->n_heads, win = c->sliding_window;
    mmq(m->qr, x, &w->attn.wq_a);
    dsv4o_rmsnorm(m->qr, m->qr, w->attn.q_norm, c->q_lora, c->rms_eps);
    mmq(m->q, m->qr, &w->attn.wq_b);
    for (int h = 0; h < H; h++) {
        float *qh = m->q + (size_t)h * hd;
        double sq = 0.0;
        for (int i = 0; i < hd; i++) sq += (double)qh[i] * qh[i];
        const float inv = (float)(1.0 / sqrt(sq / (double)hd + (double)c->rms_eps));
        for (int i = 0; i < hd; i++) qh[i] *= inv;
        dsv4o_rope_apply(qh, hd, rd, cs, sn, pos, rd / 2, 0);
    }
    mmq(m->kv, x, &w->attn.wkv);
    dsv4o_rmsnorm(m->kv, m->kv, w->attn.kv_norm, hd, c->rms_eps);
    dsv4o_rope_apply(m->kv, hd, rd, cs, sn, pos, rd / 2, 0);
    memcpy(st->kv_cache + (size_t)(pos % win) * hd, m->kv, (size_t)hd * 4);
    if (w->has_comp) {
        const int ratio = w->compress_ratio;
        mmq(m->comp_in, x, &w->attn.comp.wkv);
        mmq(m->comp_sc, x, &w->attn.comp.wgate);
        if (dsv4o_compress_step(m->kv, m->comp_in, m->comp_sc, w->attn.comp.ape, st->comp_kv, st->comp_score,
                                pos, ratio, hd)) {
            dsv4o_rmsnorm(m->kv, m->kv, w->attn.comp.norm, hd, c->rms_eps);
            dsv4o_rope_apply(m->kv, hd, rd, cs, sn, pos + 1 - ratio, rd / 2, 0);
            memcpy(st->kv_cache + (size_t)(win + st->n_compressed) * hd, m->kv, (size_t)hd * 4);
            st->n_compressed++;
        }
        const int avail = st->n_compressed;
        int take = avail;
        if (avail > 0) {
            if (w->has_idx) {
                mmq(m->idx_q, m->qr, &w->attn.idx.wq_b);
                for (int h = 0; h < c->index_n_heads; h++)
                    dsv4o_rope_apply(m->idx_q + (size_t)h * c->index_head_dim, c->index_head_dim, rd, cs, sn,
                                     pos, rd / 2, 0);
                mmq(m->idx_w, x, &w->attn.idx.weights_proj);
                /* the reference reads the compressed region as CONTIGUOUS
                 * rows of index_head_dim floats (dsv4_layer.c:286-289 with
                 * dsv4_indexer.c:71), not at the attention row stride */
                dsv4o_indexer_score_strided(m->idx_scores, m->idx_q, st->kv_cache + (size_t)win * hd,
                                            c->index_head_dim, m->idx_w, c->index_n_heads,
                                            c->index_head_dim, avail);
                take = avail < c->index_topk ? avail : c->index_topk;
                dsv4o_topk(m->idxs + n_idx, m->idx_scores, avail, take);
            } else {
                for (int i = 0; i < take; i++) m->idxs[n_idx + i] = i;
            }
            dsv4o_indexer_offset(m->idxs + n_idx, take, win);
            n_idx += take;
        }
    }
    dsv4o_sparse_attn(m->o, m->q, st->kv_cache, w->attn.sink, m->idxs, H, hd, n_idx,
                      1.0f / sqrtf((float)hd), m->attn_scratch);
    for (int h = 0; h < H; h++) dsv4o_rope_apply(m->o + (size_t)h * hd, hd, rd, cs, sn, pos, rd / 2, 1);
    const int gw = H * hd / c->o_groups, gr = c->o_lora;
    const DSV4QMat *wa = &w->attn.wo_a;
    const size_t esz = (wa->wdt == DSV4_WBF16) ? 2u : 1u;
    const size_t row_bytes = (wa->wdt == DSV4_WFP4) ? (size_t)gw / 2u : (size_t)gw * esz;
    for (int g = 0; g < c->o_groups; g++) {
        DSV4QMat slice = *wa;
        slice.rows = gr;
        slice.cols = gw;
        slice.w = (const unsigned char *)wa->w + (size_t)g * gr * row_bytes;
        if (slice.s) {
            const size_t sc_row = (size_t)((gw + slice.blk_c - 1) / slice.blk_c);
            slice.s = (const unsigned char *)wa->s + (size_t)g * (size_t)(gr / (slice.blk_r ? slice.blk_r : 1)) * sc_row;
        }
        mmq(m->ogrp + (size_t)g * gr, m->o + (size_t)g * gw, &slice);
    }
    mmq(out, m->ogrp, &w->attn.wo_b);
}

/* expert_forward, src/model/dsv4_layer.c:199-206 */
static void expert(dsv4o_model *m, float *out, const float *x, const DSV4ExpertW *e, int inter)
{
    mmq(m->eg, x, &e->w1);
    mmq(m->eu, x, &e->w3);
    dsv4o_swiglu(m->eh, m->eg, m->eu, inter, m->c.swiglu_limit);
    mmq(out, m->eh, &e->w2);
}

/* src/model/dsv4_layer.c:369-484 */
static void moe(dsv4o_model *m, float *out, const float *x, const DSV4LayerW *w, int L, int token)
{
    const DSV4Cfg *c = &m->c;
    const int d = c->hidden;
    int idx[DSV4_MAX_TOPK];
    float wts[DSV4_MAX_TOPK];
    mmq(m->gate_scores, x, &w->moe.gate);
    dsv4o_route(idx, wts, m->gate_scores, m->gate_orig, w->moe.bias, w->moe.tid2eid, token, c->n_experts,
                c->topk, c->routed_scale, c->scoring_func == DSV4_SCORE_SIGMOID ? DSV4O_SCORE_SIGMOID
                                                                              : DSV4O_SCORE_SQRTSOFTPLUS);
    for (int k = 0; k < c->topk; k++)
        expert(m, m->acc + (size_t)k * d, x, &m->ex[(size_t)L * c->n_experts + idx[k]], c->moe_inter);
    for (int i = 0; i < d; i++) out[i] = 0.0f;
    for (int k = 0; k < c->topk; k++) {
        const float wk = wts[k];
        const float *a = m->acc + (size_t)k * d;
        for (int i = 0; i < d; i++) out[i] += wk * a[i];
    }
    expert(m, m->acc, x, &w->moe.shared, c->moe_inter * c->n_shared);
    for (int i = 0; i < d; i++) out[i] += m->acc[i];
}

/* One token through the whole model (src/cli/dsv4_run.c:444-483): embed,
 * replicate hc_mult times, every layer, hc_head, final norm, head, argmax.
 * Positions must be fed in order from 0. Returns the argmax; logits (vocab)
 * are written when non-NULL. */
int dsv4o_model_step(dsv4o_model *m, int token, int pos, float *logits)
{
    const DSV4Cfg *c = &m->c;
    const int hc = c->hc_mult, d = c->hidden;
    const size_t wide = (size_t)hc * d;
    if (pos < 0 || pos >= m->max_pos) return -1;
    /* dsv4_embed_row (include/dsv4/dsv4.h:300-314) */
    if (m->mw->wdt == DSV4_WBF16) {
        const uint16_t *row = (const uint16_t *)m->mw->embed + (size_t)token * d;
        for (int i = 0; i < d; i++) m->xh[i] = dsv4o_bf16(row[i]);
    } else {
        memcpy(m->xh, (const float *)m->mw->embed + (size_t)token * d, (size_t)d * 4);
    }
    for (int j = 0; j < hc; j++) memcpy(m->h + (size_t)j * d, m->xh, (size_t)d * 4);
    for (int L = 0; L < c->n_layers; L++) {
        const DSV4LayerW *w = &m->lw[L];
        const int comp = m->ratios[L] != 0;
        const float *cs = comp ? m->cs_c : m->cs_d, *sn = comp ? m->sn_c : m->sn_d;
        memcpy(m->resid, m->h, wide * 4);
        dsv4o_hc_pre(m->x1, m->post, m->comb, m->mixes, m->h, w->hc_attn.fn, w->hc_attn.base, w->hc_attn.scale,
                     hc, d, c->hc_sinkhorn_iters, c->rms_eps, c->hc_eps);
        dsv4o_rmsnorm(m->x1, m->x1, w->attn_norm, d, c->rms_eps);
        /* window slots first; compressed selections are appended after the
         * VALID window entries (dsv4_layer.c:504-505, :291) */
        const int n_idx = dsv4o_window_idxs(m->idxs, pos, c->sliding_window);
        attention(m, m->blk, m->x1, w, &m->st[L], cs, sn, pos, n_idx);
        dsv4o_hc_post(m->h, m->blk, m->resid, m->post, m->comb, hc, d);
        memcpy(m->resid, m->h, wide * 4);
        dsv4o_hc_pre(m->x1, m->post, m->comb, m->mixes, m->h, w->hc_ffn.fn, w->hc_ffn.base, w->hc_ffn.scale,
                     hc, d, c->hc_sinkhorn_iters, c->rms_eps, c->hc_eps);
        dsv4o_rmsnorm(m->x1, m->x1, w->ffn_norm, d, c->rms_eps);
        moe(m, m->blk, m->x1, w, L, token);
        dsv4o_hc_post(m->h, m->blk, m->resid, m->post, m->comb, hc, d);
    }
    dsv4o_hc_head(m->xh, m->h, m->mw->hc_head.fn, m->mw->hc_head.base, m->mw->hc_head.scale, hc, d,
                  c->rms_eps, c->hc_eps);
    dsv4o_rmsnorm(m->xh, m->xh, m->mw->norm, d, c->rms_eps);
    DSV4QMat head = { m->mw->head, NULL, m->mw->wdt, c->vocab, d, 0, 0 };
    mmq(m->logits, m->xh, &head);
    int best = 0;
    for (int v = 1; v < c->vocab; v++) if (m->logits[v] > m->logits[best]) best = v;
    if (logits) memcpy(logits, m->logits, (size_t)c->vocab * 4);
    return best;
}

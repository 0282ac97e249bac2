/* ref_model_driver.c - greedy decode through the REFERENCE's own layer code.
 *
 * TEST INFRASTRUCTURE ONLY. Compiled with the reference's headers and linked
 * with its src/core + src/model sources (oracle/Makefile, target `ref`) into
 * _ref/libdsv4ref.so. It drives dsv4_layer_forward (src/model/dsv4_layer.c:487)
 * the way src/cli/dsv4_run.c:444-483 does, with experts served from an array
 * through DSV4ExpertSrc.get (src/model/dsv4_layer.h:46-74). The CLI's hc_head
 * is static there, so it is written out here (dsv4_run.c:94-116). Used only to
 * generate the golden token stream that pins the oracle's restated model. */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "dsv4.h"
#include "dsv4_layer.h"

void dsv4_rope_table(float *, float *, int, int, int, double, double, double, double);
void dsv4_rmsnorm(float *, const float *, const float *, int, float);
void dsv4_mmq(float *, const float *, const DSV4QMat *);

typedef struct { const DSV4ExpertW *ex; int n; } Src;

static const DSV4ExpertW *get_expert(void *ctx, int layer, int e)
{
    const Src *s = (const Src *)ctx;
    return &s->ex[(size_t)layer * s->n + e];
}

static void hc_head(float *y, const float *x, const DSV4HcW *w, int hc, int hidden, float norm_eps, float hc_eps)
{
    const int hcdim = hc * hidden;
    double sq = 0.0;
    for (int i = 0; i < hcdim; i++) sq += (double)x[i] * x[i];
    const float rs = (float)(1.0 / sqrt(sq / (double)hcdim + (double)norm_eps));
    float pre[DSV4_MAX_HC_MULT];
    for (int j = 0; j < hc; j++) {
        const float *row = w->fn + (size_t)j * hcdim;
        double acc = 0.0;
        for (int i = 0; i < hcdim; i++) acc = fma((double)row[i], (double)x[i], acc);
        const float m = (float)acc * rs;
        pre[j] = 1.0f / (1.0f + expf(-(m * w->scale[0] + w->base[j]))) + hc_eps;
    }
    for (int d = 0; d < hidden; d++) {
        double acc = 0.0;
        for (int j = 0; j < hc; j++) acc += (double)pre[j] * (double)x[(size_t)j * hidden + d];
        y[d] = (float)acc;
    }
}

static double now_s(void)
{
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

static int run(const DSV4Cfg *c, const DSV4ModelW *mw, const DSV4LayerW *lw, const DSV4ExpertW *ex, int max_pos,
               const int *tokens, int n_prompt, int n_gen, int *out_tokens, float *logits, double *t_layer,
               double *t_head)
{
    const int hc = c->hc_mult, d = c->hidden, half = c->qk_rope / 2;
    float *cs_d = malloc((size_t)max_pos * half * 4), *sn_d = malloc((size_t)max_pos * half * 4);
    float *cs_c = malloc((size_t)max_pos * half * 4), *sn_c = malloc((size_t)max_pos * half * 4);
    dsv4_rope_table(cs_d, sn_d, c->qk_rope, max_pos, 0, c->rope_theta, c->yarn_factor, c->yarn_beta_fast,
                    c->yarn_beta_slow);
    dsv4_rope_table(cs_c, sn_c, c->qk_rope, max_pos, c->yarn_orig_ctx, c->compress_rope_theta, c->yarn_factor,
                    c->yarn_beta_fast, c->yarn_beta_slow);
    DSV4Scratch s;
    if (dsv4_scratch_init(&s, c, max_pos) != 0) return -1;
    DSV4LayerState *st = calloc((size_t)c->n_layers, sizeof *st);
    for (int L = 0; L < c->n_layers; L++)
        if (dsv4_state_init(&st[L], c, L, max_pos) != 0) return -1;
    Src src = { ex, c->n_experts };
    DSV4ExpertSrc es = { get_expert, NULL, NULL, NULL, &src };
    float *h = calloc((size_t)hc * d, 4), *xh = calloc((size_t)d, 4), *lg = calloc((size_t)c->vocab, 4);
    int *ids = malloc((size_t)(n_prompt + n_gen + 1) * sizeof(int));
    memcpy(ids, tokens, (size_t)n_prompt * sizeof(int));
    int emitted = 0;
    for (int pos = 0; pos < n_prompt + n_gen && pos < max_pos; pos++) {
        const int tid = ids[pos];
        dsv4_embed_row(xh, mw->embed, mw->wdt, tid, d);
        for (int j = 0; j < hc; j++) memcpy(h + (size_t)j * d, xh, (size_t)d * 4);
        for (int L = 0; L < c->n_layers; L++) {
            const int comp = dsv4_compress_ratio(c, L) != 0;
            const double t0 = t_layer ? now_s() : 0.0;
            dsv4_layer_forward(h, &lw[L], c, &s, &es, &st[L], comp ? cs_c : cs_d, comp ? sn_c : sn_d, pos, tid);
            if (t_layer) t_layer[(size_t)pos * c->n_layers + L] = now_s() - t0;
        }
        if (pos + 1 >= n_prompt) {
            const double t0 = t_head ? now_s() : 0.0;
            hc_head(xh, h, &mw->hc_head, hc, d, c->rms_eps, c->hc_eps);
            dsv4_rmsnorm(xh, xh, mw->norm, d, c->rms_eps);
            DSV4QMat head = { mw->head, NULL, mw->wdt, c->vocab, d, 0, 0 };
            dsv4_mmq(lg, xh, &head);
            int best = 0;
            for (int v = 1; v < c->vocab; v++) if (lg[v] > lg[best]) best = v;
            ids[pos + 1] = best;
            out_tokens[emitted] = best;
            if (logits) memcpy(logits + (size_t)emitted * c->vocab, lg, (size_t)c->vocab * 4);
            emitted++;
            if (t_head) t_head[pos] = now_s() - t0;
        }
    }
    for (int L = 0; L < c->n_layers; L++) dsv4_state_free(&st[L]);
    free(st); dsv4_scratch_free(&s);
    free(cs_d); free(sn_d); free(cs_c); free(sn_c); free(h); free(xh); free(lg); free(ids);
    return emitted;
}

/* tokens[0..n_prompt) is the prompt; positions run 0..n_prompt+n_gen-1 and
 * every position from n_prompt-1 on emits a greedy token into out_tokens and
 * (if logits != NULL) its logits row. Returns the number of tokens emitted. */
int dsv4ref_greedy(const DSV4Cfg *c, const DSV4ModelW *mw, const DSV4LayerW *lw, const DSV4ExpertW *ex,
                   int max_pos, const int *tokens, int n_prompt, int n_gen, int *out_tokens, float *logits)
{
    return run(c, mw, lw, ex, max_pos, tokens, n_prompt, n_gen, out_tokens, logits, NULL, NULL);
}

/* The same loop from a one-token prompt for n_pos positions, timing each
 * layer call (t_layer[pos * n_layers + L], seconds) and each head + argmax
 * (t_head[pos]): the CPU baseline of the decode benchmark. */
int dsv4ref_decode_timed(const DSV4Cfg *c, const DSV4ModelW *mw, const DSV4LayerW *lw, const DSV4ExpertW *ex,
                         int max_pos, int first_token, int n_pos, int *out_tokens, double *t_layer, double *t_head)
{
    return run(c, mw, lw, ex, max_pos, &first_token, 1, n_pos - 1, out_tokens, NULL, t_layer, t_head);
}

/* The same timed loop after a prompt: tokens[0..n_prompt) are fed first (the
 * reference's prompt path, layer calls only), then n_gen greedy positions.
 * t_layer / t_head are indexed by position (n_prompt + n_gen rows); t_head is
 * written from position n_prompt - 1 on. The like-for-like CPU arm of the
 * decode benchmark, which times the GPU's positions after the same prompt. */
int dsv4ref_decode_timed_prompt(const DSV4Cfg *c, const DSV4ModelW *mw, const DSV4LayerW *lw,
                                const DSV4ExpertW *ex, int max_pos, const int *tokens, int n_prompt, int n_gen,
                                int *out_tokens, double *t_layer, double *t_head)
{
    return run(c, mw, lw, ex, max_pos, tokens, n_prompt, n_gen, out_tokens, NULL, t_layer, t_head);
}

/* The reference's batched prompt path (src/cli/dsv4_run.c:391-442): the
 * prompt in passes of up to chunk tokens, each pass every layer's
 * dsv4_layer_forward_n (src/model/dsv4_layer.c:856) over the pass's rows,
 * the head on the prompt's last token only, then n_gen positions of the
 * per-token loop. out_tokens receives the n_gen + 1 greedy tokens from
 * position n_prompt - 1 on (the same ones dsv4ref_greedy gives: the
 * reference gates batched against per-token bit equality); t_pass (may be
 * NULL) the seconds of each pass's layer calls, t_pass[pass * n_layers + L].
 * Returns the tokens emitted, or -1. */
int dsv4ref_prefill_greedy(const DSV4Cfg *c, const DSV4ModelW *mw, const DSV4LayerW *lw, const DSV4ExpertW *ex,
                           int max_pos, const int *tokens, int n_prompt, int n_gen, int chunk, int *out_tokens,
                           double *t_pass)
{
    if (chunk < 1 || chunk > DSV4_MAX_BATCH || n_prompt < 1 || n_prompt + n_gen > max_pos) return -1;
    const int hc = c->hc_mult, d = c->hidden, half = c->qk_rope / 2;
    const size_t wide = (size_t)hc * d;
    float *cs_d = malloc((size_t)max_pos * half * 4), *sn_d = malloc((size_t)max_pos * half * 4);
    float *cs_c = malloc((size_t)max_pos * half * 4), *sn_c = malloc((size_t)max_pos * half * 4);
    dsv4_rope_table(cs_d, sn_d, c->qk_rope, max_pos, 0, c->rope_theta, c->yarn_factor, c->yarn_beta_fast,
                    c->yarn_beta_slow);
    dsv4_rope_table(cs_c, sn_c, c->qk_rope, max_pos, c->yarn_orig_ctx, c->compress_rope_theta, c->yarn_factor,
                    c->yarn_beta_fast, c->yarn_beta_slow);
    DSV4Scratch s;
    DSV4Batch bat;
    if (dsv4_scratch_init(&s, c, max_pos) != 0) return -1;
    if (dsv4_batch_init(&bat, c, chunk) != 0) return -1;
    DSV4LayerState *st = calloc((size_t)c->n_layers, sizeof *st);
    for (int L = 0; L < c->n_layers; L++)
        if (dsv4_state_init(&st[L], c, L, max_pos) != 0) return -1;
    Src src = { ex, c->n_experts };
    DSV4ExpertSrc es = { get_expert, NULL, NULL, NULL, &src };
    float *h = calloc(wide, 4), *hb = calloc((size_t)chunk * wide, 4);
    float *xh = calloc((size_t)d, 4), *lg = calloc((size_t)c->vocab, 4);
    int32_t *tb = calloc((size_t)chunk, sizeof(int32_t));
    int *ids = malloc((size_t)(n_prompt + n_gen + 1) * sizeof(int));
    memcpy(ids, tokens, (size_t)n_prompt * sizeof(int));
    DSV4QMat head = { mw->head, NULL, mw->wdt, c->vocab, d, 0, 0 };
    int emitted = 0, pass = 0;
    for (int p0 = 0; p0 < n_prompt; p0 += chunk, pass++) {
        const int nt = n_prompt - p0 < chunk ? n_prompt - p0 : chunk;
        for (int t = 0; t < nt; t++) {
            tb[t] = ids[p0 + t];
            dsv4_embed_row(xh, mw->embed, mw->wdt, tb[t], d);
            for (int j = 0; j < hc; j++) memcpy(hb + (size_t)t * wide + (size_t)j * d, xh, (size_t)d * 4);
        }
        for (int L = 0; L < c->n_layers; L++) {
            const int comp = dsv4_compress_ratio(c, L) != 0;
            const double t0 = now_s();
            dsv4_layer_forward_n(hb, &lw[L], c, &s, &bat, &es, &st[L], comp ? cs_c : cs_d, comp ? sn_c : sn_d, p0,
                                 tb, nt);
            if (t_pass) t_pass[(size_t)pass * c->n_layers + L] = now_s() - t0;
        }
        if (p0 + nt >= n_prompt) memcpy(h, hb + (size_t)(nt - 1) * wide, wide * 4);
    }
    /* the head on the last prompt token, then the per-token loop */
    for (int pos = n_prompt - 1; pos < n_prompt + n_gen; pos++) {
        if (pos >= n_prompt) {
            const int tid = ids[pos];
            dsv4_embed_row(xh, mw->embed, mw->wdt, tid, d);
            for (int j = 0; j < hc; j++) memcpy(h + (size_t)j * d, xh, (size_t)d * 4);
            for (int L = 0; L < c->n_layers; L++) {
                const int comp = dsv4_compress_ratio(c, L) != 0;
                dsv4_layer_forward(h, &lw[L], c, &s, &es, &st[L], comp ? cs_c : cs_d, comp ? sn_c : sn_d, pos,
                                   tid);
            }
        }
        hc_head(xh, h, &mw->hc_head, hc, d, c->rms_eps, c->hc_eps);
        dsv4_rmsnorm(xh, xh, mw->norm, d, c->rms_eps);
        dsv4_mmq(lg, xh, &head);
        int best = 0;
        for (int v = 1; v < c->vocab; v++) if (lg[v] > lg[best]) best = v;
        ids[pos + 1] = best;
        out_tokens[emitted++] = best;
    }
    for (int L = 0; L < c->n_layers; L++) dsv4_state_free(&st[L]);
    free(st); dsv4_scratch_free(&s); dsv4_batch_free(&bat);
    free(cs_d); free(sn_d); free(cs_c); free(sn_c); free(h); free(hb); free(xh); free(lg); free(tb); free(ids);
    return emitted;
}

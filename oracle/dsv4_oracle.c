/* dsv4_oracle.c - CPU restatement of the deepseek-v4-in-c hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the B200 kernels, never the thing
 * measured or shipped. See dsv4_oracle.h for the rules.
 *
 * Build with -ffp-contract=off (oracle/Makefile does): the reference's
 * bit-exactness rests on every multiply and add being rounded separately
 * unless an explicit fma() says otherwise (reference Makefile:5-10).
 */
#include "dsv4_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------- formats --- */

/* src/core/dsv4_quant.h:74-88. 0xFF is NaN, 0x00 is the subnormal 2^-127. */
float dsv4o_e8m0(uint8_t b)
{
    union { uint32_t u; float f; } v;
    if (b == 0xFFu) v.u = 0x7FC00000u;
    else if (b == 0u) v.u = 0x00400000u;
    else v.u = (uint32_t)b << 23;
    return v.f;
}

/* src/core/dsv4_quant.h:101-130. Written as value arithmetic rather than bit
 * assembly: every e4m3 value is m * 2^(e-10) with an integer m, which is exact
 * in float. exp 15 / man 7 is the only NaN; there is no infinity. */
float dsv4o_e4m3(uint8_t b)
{
    const int e = (b >> 3) & 0xF, m = b & 7;
    float mag;
    if (e == 0xF && m == 7) mag = NAN;
    else if (e == 0) mag = ldexpf((float)m, -9);
    else mag = ldexpf((float)(8 + m), e - 10);
    return (b & 0x80u) ? -mag : mag;
}

/* src/core/dsv4_quant.h:141-149: magnitudes {0,.5,1,1.5,2,3,4,6}, bit 3 sign. */
float dsv4o_e2m1(uint8_t nib)
{
    static const float mag[8] = { 0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f };
    const float v = mag[nib & 7u];
    return (nib & 8u) ? -v : v;
}

float dsv4o_bf16(uint16_t h)
{
    union { uint32_t u; float f; } v;
    v.u = (uint32_t)h << 16;
    return v.f;
}

/* ---------------------------------------------------------------- GEMV --- */

/* The reduction every packed GEMV uses (src/core/dsv4_matmul.c:51-64): sixteen
 * double accumulators, lane l taking elements l, l+16, l+32, ...; folded as
 * ((a0+a4)+(a8+a12)) + ((a1+a5)+(a9+a13)) + ... ; then any tail of fewer than
 * 16 elements chained onto the result with fma in order. */
static double tree16(const double *w, const double *x, int n)
{
    double a[16];
    for (int l = 0; l < 16; l++) a[l] = 0.0;
    int i = 0;
    for (; i + 15 < n; i += 16)
        for (int l = 0; l < 16; l++) a[l] = fma(w[i + l], x[i + l], a[l]);
    const double b0 = (a[0] + a[4]) + (a[8] + a[12]);
    const double b1 = (a[1] + a[5]) + (a[9] + a[13]);
    const double b2 = (a[2] + a[6]) + (a[10] + a[14]);
    const double b3 = (a[3] + a[7]) + (a[11] + a[15]);
    double acc = (b0 + b1) + (b2 + b3);
    for (; i < n; i++) acc = fma(w[i], x[i], acc);
    return acc;
}

static double *widen(const float *x, size_t n)
{
    double *d = (double *)malloc(n * sizeof *d);
    if (!d) { fprintf(stderr, "dsv4_oracle: out of memory\n"); abort(); }
    for (size_t i = 0; i < n; i++) d[i] = (double)x[i];
    return d;
}

/* Decode element c of row `o` of a block-scaled matrix to double. */
static inline double fp8_at(const uint8_t *row, int c) { return (double)dsv4o_e4m3(row[c]); }
static inline double fp4_at(const uint8_t *row, int c)
{
    /* src/core/dsv4_quant.h:155-164: even element in the LOW nibble. */
    const uint8_t byte = row[c >> 1];
    return (double)dsv4o_e2m1((c & 1) ? (uint8_t)(byte >> 4) : (uint8_t)(byte & 15u));
}

/* One row of a block-scaled GEMV for nt tokens: dsv4_matmul.c:293-345 for nt=1
 * and :400-457 for the batched form, which per (row, token) is the same sum. */
static void scaled_row(float *y, size_t ystride, const double *xd, int in,
                       const uint8_t *row, const uint8_t *S, int o, int blk_r,
                       int blk_c, int fp4, int nt, double *wbuf)
{
    const int sc = (in + blk_c - 1) / blk_c;
    double total[64];
    for (int t = 0; t < nt; t++) total[t] = 0.0;
    for (int c0 = 0; c0 < in; c0 += blk_c) {
        const int n = (in - c0 < blk_c) ? (in - c0) : blk_c;
        for (int i = 0; i < n; i++) wbuf[i] = fp4 ? fp4_at(row, c0 + i) : fp8_at(row, c0 + i);
        const double s = (double)dsv4o_e8m0(S[(size_t)(o / blk_r) * sc + (c0 / blk_c)]);
        for (int t = 0; t < nt; t++) {
            const double acc = tree16(wbuf, xd + (size_t)t * in + c0, n);
            total[t] += acc * s;
        }
    }
    for (int t = 0; t < nt; t++) y[(size_t)t * ystride + o] = (float)total[t];
}

static void gemv_scaled(float *y, const float *x, const uint8_t *W,
                        const uint8_t *S, int in, int out, int blk_r, int blk_c,
                        int nt, int fp4)
{
    if (nt < 1 || nt > 64) { fprintf(stderr, "dsv4_oracle: nt %d\n", nt); abort(); }
    double *xd = widen(x, (size_t)in * nt);
    const size_t rb = fp4 ? (size_t)in / 2 : (size_t)in;
    #pragma omp parallel
    {
        double *wbuf = (double *)malloc((size_t)blk_c * sizeof(double));
        #pragma omp for schedule(static)
        for (int o = 0; o < out; o++)
            scaled_row(y, (size_t)out, xd, in, W + (size_t)o * rb, S, o, blk_r,
                       blk_c, fp4, nt, wbuf);
        free(wbuf);
    }
    free(xd);
}

void dsv4o_gemv_fp8(float *y, const float *x, const uint8_t *W,
                    const uint8_t *S, int in, int out, int blk_r, int blk_c)
{ gemv_scaled(y, x, W, S, in, out, blk_r, blk_c, 1, 0); }

void dsv4o_gemv_fp4(float *y, const float *x, const uint8_t *W,
                    const uint8_t *S, int in, int out, int blk_r, int blk_c)
{ gemv_scaled(y, x, W, S, in, out, blk_r, blk_c, 1, 1); }

void dsv4o_gemv_fp8_n(float *y, const float *x, const uint8_t *W,
                      const uint8_t *S, int in, int out, int blk_r, int blk_c,
                      int nt)
{ gemv_scaled(y, x, W, S, in, out, blk_r, blk_c, nt, 0); }

void dsv4o_gemv_fp4_n(float *y, const float *x, const uint8_t *W,
                      const uint8_t *S, int in, int out, int blk_r, int blk_c,
                      int nt)
{ gemv_scaled(y, x, W, S, in, out, blk_r, blk_c, nt, 1); }

/* Unscaled whole-row tree: dsv4_matmul.c:275-291 (bf16) and :380-398. */
static void gemv_plain(float *y, const float *x, const void *W, int in, int out,
                       int nt, int is_f32)
{
    double *xd = widen(x, (size_t)in * nt);
    #pragma omp parallel
    {
        double *wbuf = (double *)malloc((size_t)in * sizeof(double));
        #pragma omp for schedule(static)
        for (int o = 0; o < out; o++) {
            if (is_f32) {
                const float *row = (const float *)W + (size_t)o * in;
                for (int i = 0; i < in; i++) wbuf[i] = (double)row[i];
            } else {
                const uint16_t *row = (const uint16_t *)W + (size_t)o * in;
                for (int i = 0; i < in; i++) wbuf[i] = (double)dsv4o_bf16(row[i]);
            }
            for (int t = 0; t < nt; t++)
                y[(size_t)t * out + o] = (float)tree16(wbuf, xd + (size_t)t * in, in);
        }
        free(wbuf);
    }
    free(xd);
}

void dsv4o_gemv_bf16(float *y, const float *x, const uint16_t *W, int in, int out)
{ gemv_plain(y, x, W, in, out, 1, 0); }
void dsv4o_gemv_bf16_n(float *y, const float *x, const uint16_t *W, int in,
                       int out, int nt)
{ gemv_plain(y, x, W, in, out, nt, 0); }
void dsv4o_gemv_f32(float *y, const float *x, const float *W, int in, int out)
{ gemv_plain(y, x, W, in, out, 1, 1); }

/* src/core/dsv4_matmul.c:516-591: dispatch by storage tag. */
void dsv4o_mmq_n(float *y, const float *x, const dsv4o_mat *m, int nt)
{
    switch (m->wdt) {
    case 0: if (nt != 1) abort();
            dsv4o_gemv_f32(y, x, (const float *)m->w, m->cols, m->rows); break;
    case 1: gemv_plain(y, x, m->w, m->cols, m->rows, nt, 0); break;
    case 2: gemv_scaled(y, x, (const uint8_t *)m->w, (const uint8_t *)m->s,
                        m->cols, m->rows, m->blk_r, m->blk_c, nt, 0); break;
    case 3: gemv_scaled(y, x, (const uint8_t *)m->w, (const uint8_t *)m->s,
                        m->cols, m->rows, m->blk_r, m->blk_c, nt, 1); break;
    default: fprintf(stderr, "dsv4_oracle: wdt %d\n", m->wdt); abort();
    }
}
void dsv4o_mmq(float *y, const float *x, const dsv4o_mat *m) { dsv4o_mmq_n(y, x, m, 1); }

/* ------------------------------------------------------- elementwise --- */

/* src/core/dsv4_ops.c:25-32: double sum of squares, eps on the mean. */
void dsv4o_rmsnorm(float *y, const float *x, const float *w, int n, float eps)
{
    double sum = 0.0;
    for (int i = 0; i < n; i++) sum += (double)x[i] * (double)x[i];
    const float inv = (float)(1.0 / sqrt(sum / (double)n + (double)eps));
    for (int i = 0; i < n; i++) y[i] = w[i] * (x[i] * inv);
}

/* src/core/dsv4_ops.c:60-78: up clamped both ways, gate from above only. */
void dsv4o_swiglu(float *y, const float *gate, const float *up, int n, float limit)
{
    for (int i = 0; i < n; i++) {
        float g = gate[i], u = up[i];
        if (limit > 0.0f) {
            if (u > limit) u = limit;
            if (u < -limit) u = -limit;
            if (g > limit) g = limit;
        }
        y[i] = (g / (1.0f + expf(-g))) * u;
    }
}

/* Descending by value, ties to the lower index: the order the reference's
 * repeated-argmax selection produces (dsv4_ops.c:122-131,
 * dsv4_indexer.c:92-106). Inputs are NaN-free. */
typedef struct { float v; int i; } vi_t;
static int vi_cmp(const void *a, const void *b)
{
    const vi_t *p = (const vi_t *)a, *q = (const vi_t *)b;
    if (p->v > q->v) return -1;
    if (p->v < q->v) return 1;
    return (p->i < q->i) ? -1 : (p->i > q->i);
}

static void select_topk(int *idx, const float *v, int n, int k)
{
    vi_t *a = (vi_t *)malloc((size_t)n * sizeof *a);
    if (!a) abort();
    for (int i = 0; i < n; i++) { a[i].v = v[i]; a[i].i = i; }
    qsort(a, (size_t)n, sizeof *a, vi_cmp);
    for (int j = 0; j < k; j++) idx[j] = a[j].i;
    free(a);
}

/* src/core/dsv4_ops.c:102-141 with the score function made selectable: the
 * reference C implements sqrt(softplus) (threshold 20, :42-45); sigmoid is
 * model.py's other scoring mode as restated in tools/dsv4_ref.py:64-93. */
void dsv4o_route(int *idx, float *wts, float *scores, float *orig,
                 const float *bias, const int64_t *tid2eid, int token_id,
                 int n_experts, int topk, float route_scale, int score_func)
{
    for (int e = 0; e < n_experts; e++) {
        const float s = scores[e];
        if (score_func == DSV4O_SCORE_SIGMOID)
            orig[e] = 1.0f / (1.0f + expf(-s));
        else
            orig[e] = sqrtf((s > 20.0f) ? s : log1pf(expf(s)));
    }
    for (int e = 0; e < n_experts; e++) scores[e] = bias ? orig[e] + bias[e] : orig[e];
    if (tid2eid) {
        for (int k = 0; k < topk; k++) idx[k] = (int)tid2eid[(int64_t)token_id * topk + k];
    } else {
        select_topk(idx, scores, n_experts, topk);
    }
    double sum = 0.0;
    for (int k = 0; k < topk; k++) { wts[k] = orig[idx[k]]; sum += (double)wts[k]; }
    const float inv = (sum != 0.0) ? (float)(1.0 / sum) : 0.0f;
    for (int k = 0; k < topk; k++) wts[k] = wts[k] * inv * route_scale;
}

/* expert_forward, src/model/dsv4_layer.c:199-206. */
static void expert_fwd(float *out, const float *x, const dsv4o_mat *w1,
                       const dsv4o_mat *w3, const dsv4o_mat *w2, int inter,
                       float limit)
{
    float *g = (float *)malloc((size_t)inter * 3 * sizeof(float));
    if (!g) abort();
    float *u = g + inter, *h = u + inter;
    dsv4o_mmq(g, x, w1);
    dsv4o_mmq(u, x, w3);
    dsv4o_swiglu(h, g, u, inter, limit);
    dsv4o_mmq(out, h, w2);
    free(g);
}

/* moe(), src/model/dsv4_layer.c:369-484: router, per-k accumulators, the
 * weighted sum strictly in k order, then the shared expert added unweighted. */
void dsv4o_moe(float *out, const float *x, const dsv4o_mat *gate,
               const float *bias, const int64_t *tid2eid, int token_id,
               const dsv4o_mat *experts, const dsv4o_mat *shared,
               int n_experts, int topk, float route_scale, int score_func,
               int hidden, int inter, int inter_shared, float swiglu_limit,
               int *idx_out, float *w_out)
{
    float *scores = (float *)malloc((size_t)n_experts * 2 * sizeof(float));
    float *acc = (float *)malloc((size_t)(topk + 1) * hidden * sizeof(float));
    if (!scores || !acc) abort();
    float *orig = scores + n_experts;
    int idx[64]; float wts[64];
    dsv4o_mmq(scores, x, gate);
    dsv4o_route(idx, wts, scores, orig, bias, tid2eid, token_id, n_experts,
                topk, route_scale, score_func);
    for (int k = 0; k < topk; k++) {
        const dsv4o_mat *e = experts + (size_t)idx[k] * 3;
        expert_fwd(acc + (size_t)k * hidden, x, &e[0], &e[1], &e[2], inter,
                   swiglu_limit);
    }
    for (int i = 0; i < hidden; i++) out[i] = 0.0f;
    for (int k = 0; k < topk; k++) {
        const float wk = wts[k];
        const float *a = acc + (size_t)k * hidden;
        for (int i = 0; i < hidden; i++) out[i] += wk * a[i];
    }
    if (shared) {
        float *sh = acc + (size_t)topk * hidden;
        expert_fwd(sh, x, &shared[0], &shared[1], &shared[2], inter_shared,
                   swiglu_limit);
        for (int i = 0; i < hidden; i++) out[i] += sh[i];
    }
    if (idx_out) for (int k = 0; k < topk; k++) idx_out[k] = idx[k];
    if (w_out) for (int k = 0; k < topk; k++) w_out[k] = wts[k];
    free(scores); free(acc);
}

/* -------------------------------------------------------------- indexer --- */

/* src/core/dsv4_indexer.c:64-85: sequential double fma per head, ReLU before
 * the head weight, heads folded in order, then (float)total * scale where
 * scale = d^-1/2 * h^-1/2 in float. */
void dsv4o_indexer_score_strided(float *out, const float *q, const float *kv,
                                 int kv_stride, const float *weights,
                                 int n_heads, int head_dim, int n_pos)
{
    const float scale = (1.0f / sqrtf((float)head_dim)) * (1.0f / sqrtf((float)n_heads));
    #pragma omp parallel for schedule(static) if (n_pos > 256)
    for (int t = 0; t < n_pos; t++) {
        const float *kt = kv + (size_t)t * kv_stride;
        double total = 0.0;
        for (int h = 0; h < n_heads; h++) {
            const float *qh = q + (size_t)h * head_dim;
            double dot = 0.0;
            for (int c = 0; c < head_dim; c++) dot = fma((double)qh[c], (double)kt[c], dot);
            if (dot > 0.0) total += dot * (double)weights[h];
        }
        out[t] = (float)total * scale;
    }
}

void dsv4o_indexer_score(float *out, const float *q, const float *kv,
                         const float *weights, int n_heads, int head_dim,
                         int n_pos)
{
    dsv4o_indexer_score_strided(out, q, kv, head_dim, weights, n_heads,
                                head_dim, n_pos);
}

/* src/core/dsv4_indexer.c:92-106, restated as a sort: same output sequence
 * (descending, ties to the lower index, k clamped to n) in O(n log n). */
int dsv4o_topk(int *idxs, const float *scores, int n, int k)
{
    if (k > n) k = n;
    if (k <= 0) return 0;
    select_topk(idxs, scores, n, k);
    return k;
}

/* src/core/dsv4_indexer.c:113-123. */
void dsv4o_indexer_offset(int *idxs, int n, int offset)
{
    for (int i = 0; i < n; i++) if (idxs[i] >= 0) idxs[i] += offset;
}
int dsv4o_indexer_navail(int pos, int ratio) { return (pos + 1) / ratio; }

/* ------------------------------------------------------------ attention --- */

/* src/core/dsv4_attn.c:60-108: per head, double dot -> float * scale; max over
 * valid slots only; e = expf(s - mx); denominator in double plus the sink's
 * expf(sink - mx); numerator over valid slots in float, slot order; scaled by
 * (float)(1/denom). scratch holds h*topk floats. */
void dsv4o_sparse_attn(float *o, const float *q, const float *kv,
                       const float *sink, const int *idxs, int h, int d,
                       int topk, float scale, float *scratch)
{
    #pragma omp parallel for schedule(static) if (h > 4)
    for (int i = 0; i < h; i++) {
        float *s = scratch + (size_t)i * topk;
        const float *qi = q + (size_t)i * d;
        float mx = -INFINITY;
        for (int j = 0; j < topk; j++) {
            if (idxs[j] < 0) { s[j] = -INFINITY; continue; }
            const float *kvj = kv + (size_t)idxs[j] * d;
            double acc = 0.0;
            for (int c = 0; c < d; c++) acc = fma((double)qi[c], (double)kvj[c], acc);
            s[j] = (float)acc * scale;
            if (s[j] > mx) mx = s[j];
        }
        double denom = 0.0;
        for (int j = 0; j < topk; j++) {
            if (idxs[j] < 0) { s[j] = 0.0f; continue; }
            s[j] = expf(s[j] - mx);
            denom += (double)s[j];
        }
        denom += (double)expf(sink[i] - mx);
        float *oi = o + (size_t)i * d;
        for (int c = 0; c < d; c++) oi[c] = 0.0f;
        for (int j = 0; j < topk; j++) {
            if (idxs[j] < 0) continue;
            const float w = s[j];
            if (w == 0.0f) continue;
            const float *kvj = kv + (size_t)idxs[j] * d;
            for (int c = 0; c < d; c++) oi[c] += w * kvj[c];
        }
        const float inv = (float)(1.0 / denom);
        for (int c = 0; c < d; c++) oi[c] *= inv;
    }
}

/* src/core/dsv4_attn.c:118-127: ring slots of the last min(pos+1, win)
 * positions, newest first, -1 for unwritten slots. */
int dsv4o_window_idxs(int *idxs, int pos, int win)
{
    const int n = (pos + 1 < win) ? pos + 1 : win;
    for (int k = 0; k < win; k++) idxs[k] = (k < n) ? (pos - k) % win : -1;
    return n;
}

/* ----------------------------------------------------------------- RoPE --- */

/* src/core/dsv4_rope.c:66-99 (and the YaRN range :48-59). */
void dsv4o_rope_table(float *cs, float *sn, int dim, int seqlen,
                      int orig_seq_len, double base, double factor,
                      double beta_fast, double beta_slow)
{
    const int half = dim / 2;
    double *f = (double *)malloc((size_t)half * sizeof(double));
    if (!f) abort();
    for (int i = 0; i < half; i++) f[i] = 1.0 / pow(base, (double)(2 * i) / (double)dim);
    if (orig_seq_len > 0) {
        const double twopi = 2.0 * 3.14159265358979323846;
        const double lo_d = (double)dim * log((double)orig_seq_len / (beta_fast * twopi)) / (2.0 * log(base));
        const double hi_d = (double)dim * log((double)orig_seq_len / (beta_slow * twopi)) / (2.0 * log(base));
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
    free(f);
}

/* src/core/dsv4_rope.c:106-120: interleaved pairs in the last rd dims;
 * inverse negates the sine. */
void dsv4o_rope_apply(float *v, int head_dim, int rd, const float *cs,
                      const float *sn, int pos, int table_half, int inverse)
{
    float *tail = v + (head_dim - rd);
    const float *c = cs + (size_t)pos * table_half;
    const float *s = sn + (size_t)pos * table_half;
    const float sgn = inverse ? -1.0f : 1.0f;
    for (int i = 0; i < rd / 2; i++) {
        const float re = tail[2 * i], im = tail[2 * i + 1];
        const float ci = c[i], si = sgn * s[i];
        tail[2 * i] = re * ci - im * si;
        tail[2 * i + 1] = re * si + im * ci;
    }
}

/* ------------------------------------------------------------------ mHC --- */

static float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

/* src/core/dsv4_hc.c:50-102: pre (+eps), post (x2), comb; first pass is a
 * row softmax +eps then a column normalise; then iters-1 row/col passes. */
void dsv4o_hc_split_sinkhorn(float *pre, float *post, float *comb,
                             const float *mixes, const float *hc_scale,
                             const float *hc_base, int hc, int iters, float eps)
{
    for (int j = 0; j < hc; j++) pre[j] = sigm(mixes[j] * hc_scale[0] + hc_base[j]) + eps;
    for (int j = 0; j < hc; j++) post[j] = 2.0f * sigm(mixes[j + hc] * hc_scale[1] + hc_base[j + hc]);
    for (int j = 0; j < hc; j++)
        for (int k = 0; k < hc; k++) {
            const int o = j * hc + k + hc * 2;
            comb[j * hc + k] = mixes[o] * hc_scale[2] + hc_base[o];
        }
    for (int j = 0; j < hc; j++) {
        float *r = comb + j * hc;
        float mx = r[0];
        for (int k = 1; k < hc; k++) if (r[k] > mx) mx = r[k];
        double sum = 0.0;
        for (int k = 0; k < hc; k++) { r[k] = expf(r[k] - mx); sum += (double)r[k]; }
        const float inv = (float)(1.0 / sum);
        for (int k = 0; k < hc; k++) r[k] = r[k] * inv + eps;
    }
    /* pass 0 is the column normalise of the first pass; the remaining
     * iters-1 passes are row then column. */
    const int npass = iters > 1 ? iters : 1;
    for (int pass = 0; pass < npass; pass++) {
        if (pass > 0)
            for (int j = 0; j < hc; j++) {
                double rs = 0.0;
                for (int k = 0; k < hc; k++) rs += (double)comb[j * hc + k];
                const float d = (float)rs + eps;
                for (int k = 0; k < hc; k++) comb[j * hc + k] /= d;
            }
        for (int k = 0; k < hc; k++) {
            double cs = 0.0;
            for (int j = 0; j < hc; j++) cs += (double)comb[j * hc + k];
            const float d = (float)cs + eps;
            for (int j = 0; j < hc; j++) comb[j * hc + k] /= d;
        }
    }
}

/* src/core/dsv4_hc.c:111-141: rsqrt over the whole flattened hc*hidden vector
 * with norm_eps, mixes = (float)(double dot) * rsqrt, then y = sum_j pre[j]x[j]
 * in double. */
void dsv4o_hc_pre(float *y, float *post, float *comb, float *mixes,
                  const float *x, const float *fn, const float *base,
                  const float *scale, int hc, int hidden, int iters,
                  float norm_eps, float hc_eps)
{
    const int hcdim = hc * hidden, mix_hc = (2 + hc) * hc;
    double sq = 0.0;
    for (int i = 0; i < hcdim; i++) sq += (double)x[i] * (double)x[i];
    const float rs = (float)(1.0 / sqrt(sq / (double)hcdim + (double)norm_eps));
    for (int m = 0; m < mix_hc; m++) {
        const float *row = fn + (size_t)m * hcdim;
        double acc = 0.0;
        for (int i = 0; i < hcdim; i++) acc = fma((double)row[i], (double)x[i], acc);
        mixes[m] = (float)acc * rs;
    }
    float pre[16];
    dsv4o_hc_split_sinkhorn(pre, post, comb, mixes, scale, base, hc, iters, hc_eps);
    for (int d = 0; d < hidden; d++) {
        double acc = 0.0;
        for (int j = 0; j < hc; j++) acc += (double)pre[j] * (double)x[(size_t)j * hidden + d];
        y[d] = (float)acc;
    }
}

/* src/core/dsv4_hc.c:149-162: y[k] = post[k]*x + sum_j comb[j][k]*res[j]. */
void dsv4o_hc_post(float *y, const float *x, const float *residual,
                   const float *post, const float *comb, int hc, int hidden)
{
    for (int k = 0; k < hc; k++)
        for (int d = 0; d < hidden; d++) {
            double acc = (double)post[k] * (double)x[d];
            for (int j = 0; j < hc; j++)
                acc += (double)comb[j * hc + k] * (double)residual[(size_t)j * hidden + d];
            y[(size_t)k * hidden + d] = (float)acc;
        }
}

/* src/cli/dsv4_run.c:94-116: sigmoid gate per copy (+eps), one scalar scale. */
void dsv4o_hc_head(float *y, const float *x, const float *fn,
                   const float *base, const float *scale, int hc, int hidden,
                   float norm_eps, float hc_eps)
{
    const int hcdim = hc * hidden;
    double sq = 0.0;
    for (int i = 0; i < hcdim; i++) sq += (double)x[i] * (double)x[i];
    const float rs = (float)(1.0 / sqrt(sq / (double)hcdim + (double)norm_eps));
    float pre[16];
    for (int j = 0; j < hc; j++) {
        const float *row = fn + (size_t)j * hcdim;
        double acc = 0.0;
        for (int i = 0; i < hcdim; i++) acc = fma((double)row[i], (double)x[i], acc);
        const float m = (float)acc * rs;
        pre[j] = 1.0f / (1.0f + expf(-(m * scale[0] + base[j]))) + hc_eps;
    }
    for (int d = 0; d < hidden; d++) {
        double acc = 0.0;
        for (int j = 0; j < hc; j++) acc += (double)pre[j] * (double)x[(size_t)j * hidden + d];
        y[d] = (float)acc;
    }
}

/* ----------------------------------------------------------- compressor --- */

/* Softmax over the slot axis for one channel (src/core/dsv4_compress.c:45-64);
 * -inf marks an unfilled slot. */
static float pool(const float *kv, const float *sc, int slots, int stride, int c)
{
    float mx = -INFINITY;
    for (int s = 0; s < slots; s++) if (sc[(size_t)s * stride + c] > mx) mx = sc[(size_t)s * stride + c];
    if (mx == -INFINITY) return 0.0f;
    double den = 0.0, acc = 0.0;
    for (int s = 0; s < slots; s++) {
        const float v = sc[(size_t)s * stride + c];
        if (v == -INFINITY) continue;
        const double e = (double)expf(v - mx);
        den += e;
        acc += e * (double)kv[(size_t)s * stride + c];
    }
    return (float)(acc / den);
}

/* src/core/dsv4_compress.c:78-138. Overlap mode (ratio 4) pools the previous
 * window's first half-width with the current window's second half-width and
 * then slides the state. */
int dsv4o_compress_step(float *out, const float *kv_in, const float *score_in,
                        const float *ape, float *kv_state, float *score_state,
                        int pos, int ratio, int head_dim)
{
    const int overlap = (ratio == 4), coff = 1 + overlap;
    const int width = coff * head_dim, phase = pos % ratio;
    const float *apr = ape + (size_t)phase * width;
    const int slot = overlap ? ratio + phase : phase;
    for (int c = 0; c < width; c++) {
        kv_state[(size_t)slot * width + c] = kv_in[c];
        score_state[(size_t)slot * width + c] = score_in[c] + apr[c];
    }
    if ((pos + 1) % ratio != 0) return 0;
    if (!overlap) {
        for (int c = 0; c < head_dim; c++)
            out[c] = pool(kv_state, score_state, ratio, width, c);
        return 1;
    }
    const int d = head_dim, ns = 2 * ratio;
    float *gk = (float *)malloc((size_t)ns * d * 2 * sizeof(float));
    if (!gk) abort();
    float *gs = gk + (size_t)ns * d;
    for (int s = 0; s < ratio; s++) {
        memcpy(gk + (size_t)s * d, kv_state + (size_t)s * width, (size_t)d * sizeof(float));
        memcpy(gs + (size_t)s * d, score_state + (size_t)s * width, (size_t)d * sizeof(float));
        memcpy(gk + (size_t)(ratio + s) * d, kv_state + (size_t)(ratio + s) * width + d, (size_t)d * sizeof(float));
        memcpy(gs + (size_t)(ratio + s) * d, score_state + (size_t)(ratio + s) * width + d, (size_t)d * sizeof(float));
    }
    for (int c = 0; c < d; c++) out[c] = pool(gk, gs, ns, d, c);
    free(gk);
    memmove(kv_state, kv_state + (size_t)ratio * width, (size_t)ratio * width * sizeof(float));
    memmove(score_state, score_state + (size_t)ratio * width, (size_t)ratio * width * sizeof(float));
    return 1;
}

/* dsv4_oracle.h - CPU restatement of the deepseek-v4-in-c decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the B200 kernels
 * are compared against. Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg may load it. The product (libdsv4_b200.so) never links or
 * calls it, and has no CPU fallback of any kind.
 *
 * Every function restates one reference function and keeps its reduction
 * order, so that on identical inputs the results are bit-identical to the
 * reference's scalar (and therefore also its AVX2) path. Each one cites the
 * reference file:line it follows. Pinned against the reference itself: the
 * golden vectors under tests/golden/ were produced by the reference's own C
 * compiled from its sources (oracle/Makefile, target `ref`), and
 * tests/test_oracle_golden.py requires bit equality.
 */
#ifndef DSV4_ORACLE_H
#define DSV4_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- numeric formats: src/core/dsv4_quant.h:74-164 ---- */
float dsv4o_e8m0(uint8_t b);
float dsv4o_e4m3(uint8_t b);
float dsv4o_e2m1(uint8_t nibble);
float dsv4o_bf16(uint16_t h);

/* ---- GEMV / batched GEMV: src/core/dsv4_matmul.c:51-64, 273-457 ----
 * y[o] = sum over blocks of (16-lane double tree of w*x) * scale, folded in
 * column order, rounded to float once. Batched forms take x [nt][in] and
 * write y [nt][out]; per (row, token) they are the GEMV exactly. */
void dsv4o_gemv_fp8(float *y, const float *x, const uint8_t *W,
                    const uint8_t *S, int in, int out, int blk_r, int blk_c);
void dsv4o_gemv_fp4(float *y, const float *x, const uint8_t *W,
                    const uint8_t *S, int in, int out, int blk_r, int blk_c);
void dsv4o_gemv_bf16(float *y, const float *x, const uint16_t *W,
                     int in, int out);
/* No F32 kernel exists in the reference (dsv4_mmq aborts on DSV4_WF32,
 * dsv4_matmul.c:539-545). This is the BF16 whole-row tree over f32 loads,
 * which is what an F32 case of that dispatch would be. */
void dsv4o_gemv_f32(float *y, const float *x, const float *W, int in, int out);
void dsv4o_gemv_fp8_n(float *y, const float *x, const uint8_t *W,
                      const uint8_t *S, int in, int out, int blk_r, int blk_c,
                      int nt);
void dsv4o_gemv_fp4_n(float *y, const float *x, const uint8_t *W,
                      const uint8_t *S, int in, int out, int blk_r, int blk_c,
                      int nt);
void dsv4o_gemv_bf16_n(float *y, const float *x, const uint16_t *W,
                       int in, int out, int nt);

/* ---- elementwise + router: src/core/dsv4_ops.c ---- */
void dsv4o_rmsnorm(float *y, const float *x, const float *w, int n, float eps);
void dsv4o_swiglu(float *y, const float *gate, const float *up, int n,
                  float limit);
enum { DSV4O_SCORE_SQRTSOFTPLUS = 1, DSV4O_SCORE_SIGMOID = 2 };
void dsv4o_route(int *idx, float *wts, float *scores, float *orig,
                 const float *bias, const int64_t *tid2eid, int token_id,
                 int n_experts, int topk, float route_scale, int score_func);

/* ---- MoE for one token: src/model/dsv4_layer.c:199-206, 369-484 ----
 * Matrix descriptors are the reference's DSV4QMat fields flattened. */
typedef struct {
    const void *w;
    const void *s;
    int wdt;                 /* 0 f32, 1 bf16, 2 fp8, 3 fp4 (dsv4.h:92) */
    int rows, cols, blk_r, blk_c;
} dsv4o_mat;
void dsv4o_mmq(float *y, const float *x, const dsv4o_mat *m);
void dsv4o_mmq_n(float *y, const float *x, const dsv4o_mat *m, int nt);
/* experts: n_experts entries of 3 matrices {w1, w3, w2}. Returns nothing;
 * idx_out/w_out receive the routing decision when not NULL. */
void dsv4o_moe(float *out, const float *x, const dsv4o_mat *gate,
               const float *bias, const int64_t *tid2eid, int token_id,
               const dsv4o_mat *experts, const dsv4o_mat *shared,
               int n_experts, int topk, float route_scale, int score_func,
               int hidden, int inter, int inter_shared, float swiglu_limit,
               int *idx_out, float *w_out);

/* ---- CSA indexer: src/core/dsv4_indexer.c:64-123 ---- */
void dsv4o_indexer_score(float *out, const float *q, const float *kv,
                         const float *weights, int n_heads, int head_dim,
                         int n_pos);
/* Same arithmetic with an explicit key row stride (floats) -- the reference
 * layer scores the attention cache at stride head_dim (dsv4_layer.c:286). */
void dsv4o_indexer_score_strided(float *out, const float *q, const float *kv,
                                 int kv_stride, const float *weights,
                                 int n_heads, int head_dim, int n_pos);
int  dsv4o_topk(int *idxs, const float *scores, int n, int k);
void dsv4o_indexer_offset(int *idxs, int n, int offset);
int  dsv4o_indexer_navail(int pos, int ratio);

/* ---- sparse attention: src/core/dsv4_attn.c:60-128 ---- */
void dsv4o_sparse_attn(float *o, const float *q, const float *kv,
                       const float *sink, const int *idxs, int h, int d,
                       int topk, float scale, float *scratch);
int  dsv4o_window_idxs(int *idxs, int pos, int win);

/* ---- RoPE: src/core/dsv4_rope.c:66-120 ---- */
void dsv4o_rope_table(float *cs, float *sn, int dim, int seqlen,
                      int orig_seq_len, double base, double factor,
                      double beta_fast, double beta_slow);
void dsv4o_rope_apply(float *v, int head_dim, int rd, const float *cs,
                      const float *sn, int pos, int table_half, int inverse);

/* ---- mHC: src/core/dsv4_hc.c:50-162, src/cli/dsv4_run.c:94-116 ---- */
void dsv4o_hc_split_sinkhorn(float *pre, float *post, float *comb,
                             const float *mixes, const float *hc_scale,
                             const float *hc_base, int hc, int iters,
                             float eps);
void dsv4o_hc_pre(float *y, float *post, float *comb, float *mixes,
                  const float *x, const float *fn, const float *base,
                  const float *scale, int hc, int hidden, int iters,
                  float norm_eps, float hc_eps);
void dsv4o_hc_post(float *y, const float *x, const float *residual,
                   const float *post, const float *comb, int hc, int hidden);
void dsv4o_hc_head(float *y, const float *x, const float *fn,
                   const float *base, const float *scale, int hc, int hidden,
                   float norm_eps, float hc_eps);

/* ---- HCA compressor: src/core/dsv4_compress.c:45-142 ---- */
int dsv4o_compress_step(float *out, const float *kv_in, const float *score_in,
                        const float *ape, float *kv_state, float *score_state,
                        int pos, int ratio, int head_dim);

/* ---- whole-token decode over the reference's structs (dsv4_oracle_model.c) ----
 * Declared with opaque pointers so this header does not need dsv4_types.h. */
typedef struct dsv4o_model dsv4o_model;
dsv4o_model *dsv4o_model_create(const void *cfg, const void *mw, const void *layers,
                                const void *experts, int max_pos);
int dsv4o_model_step(dsv4o_model *m, int token, int pos, float *logits);
void dsv4o_model_free(dsv4o_model *m);

#ifdef __cplusplus
}
#endif
#endif

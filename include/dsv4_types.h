/* dsv4_types.h - the reference's model-level types, layout-identical.
 *
 * These are include/dsv4/dsv4.h:94-295 of deepseek-v4-in-c (DSV4Cfg,
 * DSV4QMat, DSV4CompressorW, DSV4IndexerW, DSV4AttnW, DSV4ExpertW, DSV4MoeW,
 * DSV4HcW, DSV4LayerW, DSV4ModelW) restated field for field, so the structs the
 * reference's binder fills can be handed to this backend unchanged. When the
 * reference's dsv4.h is included first (DSV4_H defined), its own definitions
 * are used instead and nothing here is declared.
 */
#ifndef DSV4_TYPES_H
#define DSV4_TYPES_H

#include <stddef.h>
#include <stdint.h>

#ifndef DSV4_H

#define DSV4_MAX_TOPK 16
#define DSV4_MAX_BATCH 64
#define DSV4_MAX_LAYERS 128
#define DSV4_MAX_HC_MULT 8

enum { DSV4_SCORE_SQRTSOFTPLUS = 1, DSV4_SCORE_SIGMOID = 2, DSV4_SCORE_SOFTMAX = 3 };
enum { DSV4_TOPK_NOAUX_TC = 1, DSV4_TOPK_GREEDY = 2 };
enum { DSV4_WF32 = 0, DSV4_WBF16 = 1, DSV4_WFP8 = 2, DSV4_WFP4 = 3 };

typedef struct {
    int hidden, n_layers, vocab;
    float rms_eps;
    int max_pos;
    int n_heads, n_kv_heads, head_dim, q_lora, o_lora, o_groups, qk_rope, sliding_window;
    int index_n_heads, index_head_dim, index_topk;
    int n_compress;
    int *compress_ratios;
    float compress_rope_theta;
    int hc_mult, hc_sinkhorn_iters;
    float hc_eps;
    int n_experts, topk, n_shared, moe_inter;
    float routed_scale;
    int norm_topk, scoring_func, topk_method;
    float swiglu_limit;
    float rope_theta, yarn_factor, yarn_beta_fast, yarn_beta_slow;
    int yarn_orig_ctx;
    int wblock_m, wblock_n;
    int num_hash_layers, num_nextn_predict;
} DSV4Cfg;

typedef struct {
    const void *w;
    const void *s;
    int wdt;
    int rows, cols;
    int blk_r, blk_c;
} DSV4QMat;

typedef struct {
    const float *ape;       /* [ratio][coff*head_dim]          */
    const float *norm;      /* [head_dim]                      */
    DSV4QMat wkv, wgate;    /* [coff*head_dim][hidden]         */
    int ratio, coff;
} DSV4CompressorW;

typedef struct {
    DSV4QMat wq_b;          /* [index_n_heads*index_head_dim][q_lora] */
    DSV4QMat weights_proj;  /* [index_n_heads][hidden]                */
    DSV4CompressorW comp;   /* bound but unused by the forward pass   */
} DSV4IndexerW;

typedef struct {
    const float *sink, *q_norm, *kv_norm;
    DSV4QMat wq_a, wq_b, wkv, wo_a, wo_b;
    DSV4CompressorW comp;
    DSV4IndexerW idx;
    int has_comp, has_idx;
} DSV4AttnW;

typedef struct {
    DSV4QMat w1, w3, w2;
} DSV4ExpertW;

typedef struct {
    DSV4QMat gate;
    const float *bias;
    const int64_t *tid2eid;
    DSV4ExpertW shared;
} DSV4MoeW;

typedef struct {
    const float *fn, *base, *scale;
} DSV4HcW;

typedef struct {
    const float *attn_norm, *ffn_norm;
    DSV4AttnW attn;
    DSV4MoeW moe;
    DSV4HcW hc_attn, hc_ffn;
    int layer, compress_ratio, hash_routed, has_comp, has_idx;
} DSV4LayerW;

typedef struct {
    const void *embed, *head;
    const float *norm;
    DSV4HcW hc_head;
    int wdt;
} DSV4ModelW;

#endif /* DSV4_H */
#endif /* DSV4_TYPES_H */

// model.h - device-resident whole-token decode (model.cu, model_kernels.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "moe.h"

#define DSV4B_MAX_HC 8
#define DSV4B_MAX_SEQ 64     // sequences of a batched model
#define DSV4B_MAX_PREFILL 64 // tokens of one prefill pass (a one-sequence model)

namespace dsv4b {

// The step a graph replay runs: token at position pos. The last kernel of a
// step writes the next one (the prompt's token while prompt remains, else
// the argmax).
struct StepState {
    int token;
    int pos;
};

__global__ void k_embed(float *h, const void *table, int wdt, const StepState *st, int hidden, int hc);
__global__ void k_hc_mix(float *mixes, const float *fn, const float *x, int n, float eps);
__global__ void k_hc_finish(float *y, float *post, float *comb, const float *mixes, const float *x,
                            const float *scale, const float *base, int hc, int hidden, int iters, float eps);
constexpr int kHcPreMixMax = 24;   // (2 + hc) * hc for hc <= 4
constexpr int kHcPreBlocks = 64;
constexpr int kHcPreYPT = 8;       // float4 columns of y per thread: hidden <= 256 * 4 * 8
// Arguments of one fused mHC launch (k_hc_pre). With blk or acc set it first
// finishes the previous sub-layer's post-mix into xout and then mixes xout;
// otherwise it mixes x. Head mode: post and comb null, nmix = hc.
struct HcPreArgs {
    float *y, *post, *comb;          // x1 (normalised), the split's post / comb
    const float *x;                  // the residual (the previous one when stepping)
    float *xout;                     // stepping: the new residual
    const float *blk;                // stepping: the sub-layer's output, or
    const float *acc, *wts, *accs;   //   an MoE's: sum_k wts[k] acc[k] (+ accs)
    const float *post_in, *comb_in;  // stepping: the previous split
    const float *fn, *scale, *base, *norm_w;
    double *part;
    unsigned *count;
    int hc, hidden, iters, nmix, topk;
    float hc_eps, rms_eps;
    // a batch: sequence blockIdx.y reads and writes its own rows (residuals
    // hc hidden apart, y / blk hidden apart, post / comb DSV4B_MAX_HC /
    // DSV4B_MAX_HC^2 apart, part gridDim.x (nmix + 1) apart, count 1 apart)
    // and its MoE scratch (acc, wts, accs) s_ms floats apart
    long s_ms;
};
// k_hc_pre: one sequence; k_hc_pre_batch: sequence blockIdx.y of a batch
__global__ void k_hc_pre(const __grid_constant__ HcPreArgs a);
__global__ void k_hc_pre_batch(const __grid_constant__ HcPreArgs a);
// a batch in two launches: the partials of every (256 columns, sequence), then
// one block per sequence for the rest (same arithmetic)
__global__ void k_hc_part_batch(const __grid_constant__ HcPreArgs a);
__global__ void k_hc_tail_batch(const __grid_constant__ HcPreArgs a);
__global__ void k_hc_head_finish(float *y, const float *mixes, const float *x, const float *scale,
                                 const float *base, int hc, int hidden, float eps);
__global__ void k_hc_post(float *y, const float *x, const float *res, const float *post, const float *comb,
                          int hc, int hidden);
__global__ void k_rmsnorm(float *y, const float *x, const float *w, int n, float eps);
// Arguments of k_attn_prep (the tasks between the q projections and the
// indexer / attention of one layer).
struct PrepArgs {
    float *q, *kv, *cache, *comp_kv, *comp_score, *idx_q;
    const float *kv_norm, *comp_in, *comp_sc, *ape, *cnorm, *cs, *sn;
    const StepState *st;
    int *dyn, *idxs;
    int H, hd, rd, win, has_comp, has_idx, ratio, index_topk, ih, id, nidx;
    float eps;
    // a batch (blockIdx.y = sequence): the caches and compressor windows of
    // consecutive sequences are s_cache / s_comp floats apart; q, kv, idx_q,
    // comp_in / comp_sc (2 hd), idxs (nidx) and st are packed per sequence
    long s_cache, s_comp;
    // a prefill pass (pass_nt > 0, blockIdx.y = token, one cache): token y's
    // KV row goes to staging row stage + y, its compressed-row counts to
    // dyn + 2 y, the compressed row it closes (if any) to the cache; the
    // compressor state moves past the pass in k_stage_commit
    int stage, pass_nt;
};
__global__ void k_attn_prep(const __grid_constant__ PrepArgs a);
__global__ void k_build_idxs(int *idxs, int nmax, const StepState *st, int win, int has_comp, int has_idx,
                             const int *dyn, const int *sel, int sel_stride, int dyn_stride, int stage);
__global__ void k_stage_commit(const __grid_constant__ PrepArgs a);
// argmax partials per sequence (k_argmax_part's blocks, <= kArgmaxParts)
constexpr int kArgmaxParts = 1024;
__global__ void k_argmax_part(float *pv, int *pi, const float *x, int n);
__global__ void k_argmax_final(StepState *st, int *out_tokens, const float *pv, const int *pi, int nparts,
                               int stride, const int *prompt, int n_prompt, unsigned *stepseq, int seq_tokens);
__global__ void k_argmax_pair(float *pair, const float *pv, const int *pi, int nparts, int offset);

__global__ void k_synth(void *dst, size_t n, int kind, float a, float b, uint64_t key);
__global__ void k_synth_slice(void *dst, int nrows, int ncols, int kind, float a, float b, uint64_t key,
                              size_t base, size_t gstride);
__global__ void k_synth_experts(uint8_t *dst, int n_experts, int hidden, int inter, int i0, int il, float b,
                                uint64_t key);
__global__ void k_synth_tid2eid(int64_t *t, int vocab, int topk, int n_experts, uint64_t key);

}  // namespace dsv4b

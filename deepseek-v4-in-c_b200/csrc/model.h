// model.h - device-resident whole-token decode (model.cu, model_kernels.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "moe.h"

#define DSV4B_MAX_HC 8

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
__global__ void k_hc_pre(float *y, float *post, float *comb, const float *x, const float *fn, const float *scale,
                         const float *base, const float *norm_w, double *part, unsigned *count, int hc, int hidden,
                         int iters, float hc_eps, float rms_eps);
__global__ void k_hc_head_finish(float *y, const float *mixes, const float *x, const float *scale,
                                 const float *base, int hc, int hidden, float eps);
__global__ void k_hc_post(float *y, const float *x, const float *res, const float *post, const float *comb,
                          int hc, int hidden);
__global__ void k_rmsnorm(float *y, const float *x, const float *w, int n, float eps);
__global__ void k_heads_norm_rope(float *v, int width, int rd, const float *cs, const float *sn,
                                  const StepState *st, int pos_off, int inverse, int do_norm, float eps);
__global__ void k_kv_finish(float *kv, const float *w, int hd, int rd, const float *cs, const float *sn,
                            const StepState *st, float eps, float *cache, int win);
__global__ void k_compress(float *cache, float *kv_state, float *score_state, const float *kv_in,
                           const float *sc_in, const float *ape, const float *norm, int ratio, int hd, int rd,
                           const float *cs, const float *sn, const StepState *st, float eps, int win,
                           int index_topk, int *dyn);
__global__ void k_build_idxs(int *idxs, int nmax, const StepState *st, int win, int has_comp, int has_idx,
                             const int *dyn, const int *sel);
__global__ void k_argmax_part(float *pv, int *pi, const float *x, int n);
__global__ void k_argmax_final(StepState *st, int *out_tokens, const float *pv, const int *pi, int nparts,
                               const int *prompt, int n_prompt);

__global__ void k_synth(void *dst, size_t n, int kind, float a, float b, uint64_t key);
__global__ void k_synth_tid2eid(int64_t *t, int vocab, int topk, int n_experts, uint64_t key);

}  // namespace dsv4b

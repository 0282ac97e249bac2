// moe.h - device-side MoE layer description shared by moe.cu, the model and
// the C ABI.
#pragma once

#include "internal.h"

#include <cuda_runtime.h>
#include <stdint.h>

namespace dsv4b {

constexpr int kMoeMaxExperts = 1024;
constexpr int kMoeMaxTopk = 16;

// A device-resident matrix in one of the checkpoint formats.
struct DevMat {
    const uint8_t *w, *s;
    int wdt, rows, cols, blk_r, blk_c;
    int f16s;                       // FP4: every scale f16-safe (gemv_mma_shape)
};

struct MoeLayer {
    DevMat gate;                    // router [n_experts][hidden]
    const float *bias;              // [n_experts] or nullptr (selection only)
    const int64_t *tid2eid;         // [vocab][topk] or nullptr: hash routing
    const int *fixed;               // [topk] experts given by the caller, or nullptr
    // routed experts: device pointer tables indexed by expert id
    const uint8_t *const *w1tab, *const *s1tab;
    const uint8_t *const *w3tab, *const *s3tab;
    const uint8_t *const *w2tab, *const *s2tab;
    int efmt, eblk_r, eblk_c;
    int ef16s;                      // FP4 experts: every scale f16-safe
    DevMat sh[3];                   // shared expert w1, w3, w2
    int has_shared;
    int n_experts, topk, hidden, inter, inter_shared, score_func;
    float route_scale, swiglu_limit;
    // sharded over GPUs, inter and inter_shared are this rank's slices of
    // every expert (moe_forward then sums the per-slot outputs across ranks)
};

struct MoeScratch {
    float *logits, *g, *u, *h, *acc, *wts;
    int *sel;
};

// out = the MoE of x. With combine false the last step (out = sum_k wts[k]
// acc[k] + the shared expert's acc) is left to the caller, which reads
// S.acc / S.wts itself (the decode step folds it into the next mHC launch).
// ex (sharded decode): where the per-slot partial outputs are summed across
// ranks before the combine; null on one GPU.
// A batch of nseq tokens (combine false, ex null): token b's x at x + b s_x,
// its scratch S shifted by b s_ms floats, its token id at token + b
// tok_stride; every token's experts and arithmetic are those of a batch-1
// call. perm (device, 5 nseq topk ints), when given, holds the batch's
// expert groups: every distinct expert's tokens, up to four to a routed item.
int moe_forward(const MoeLayer &L, const MoeScratch &S, float *out, const float *x,
                const int *token, cudaStream_t st, bool combine = true, const Exch *ex = nullptr, int nseq = 1,
                long s_ms = 0, long s_x = 0, int tok_stride = 0, int *perm = nullptr);
size_t moe_scratch_floats(int hidden, int inter, int inter_shared, int n_experts, int topk);
void moe_scratch_carve(MoeScratch &S, float *base, int hidden, int inter, int inter_shared,
                       int n_experts, int topk);

}  // namespace dsv4b

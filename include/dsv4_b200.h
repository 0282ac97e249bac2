/* dsv4_b200.h - C ABI of the B200 (sm_100a) decode backend for deepseek-v4-in-c.
 *
 * Two layers, both plain C (pointers and sizes, no CUDA or torch types):
 *
 * 1. THE DROP-IN. Every symbol the reference host calls through
 *    include/dsv4/dsv4_cuda.h, with the same names, arguments, 0/-1 returns and
 *    abort-on-misuse, so libdsv4_b200.so links in place of the reference's
 *    build/dsv4_cuda.o (reference Makefile:148-160). Widened where the
 *    reference stops short: uploads accept FP8, FP4, BF16 and F32 (it accepts
 *    FP8 only, dsv4_cuda.cu:310), and a matrix whose rows lie inside a
 *    resident matrix -- the grouped wo_a slices of dsv4_layer.c:321-334 -- runs
 *    on the device instead of silently falling back to the CPU.
 *    Host-buffer twins of the reference's CPU kernels on the hot path
 *    (router, expert FFN, indexer, top-k, sparse attention) follow, each with
 *    the argument meaning of the function it replaces.
 *
 * 2. THE DEVICE API (dsv4b_*). The same kernels on device pointers, enqueued
 *    on a caller stream (a cudaStream_t passed as void*; NULL = the backend's
 *    own stream), never synchronising, so a whole decode step can be captured
 *    in a CUDA graph.
 *
 * Weight formats are the checkpoint's (reference src/core/dsv4_quant.h):
 * wdt 0 = F32, 1 = BF16, 2 = FP8 e4m3 + E8M0 blocks (128x128), 3 = FP4 e2m1
 * packed two per byte (even element in the low nibble) + E8M0 1x32 blocks.
 */
#ifndef DSV4_B200_H
#define DSV4_B200_H

#include <stddef.h>
#include <stdint.h>

/* DSV4QMat, DSV4Cfg, DSV4LayerW, ... : the reference's own types, mirrored
 * layout-identically (include/dsv4/dsv4.h:94-295), so pointers to the structs
 * the reference's binder fills pass straight through. */
#include "dsv4_types.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ===================================================== 1. the drop-in ===== */

/* include/dsv4/dsv4_cuda.h:65 -- 1 when a CUDA device is present. */
int dsv4_cuda_available(void);

/* include/dsv4/dsv4_cuda.h:70 -- bring up device 0 (or $DSV4_DEVICE); prints
 * the device and free HBM. 0 on success, -1 on failure. */
int dsv4_cuda_init(void);

/* src/cuda/dsv4_cuda.cu:264 -- choose blocking sync; call before init. */
int dsv4_cuda_set_blocking_sync(void);

/* include/dsv4/dsv4_cuda.h:80 -- copy one matrix to HBM, keyed by its host
 * weight pointer. 0 on success (or already resident), -1 = keep it on the CPU
 * (recoverable: no device, would not fit, unsupported format). */
int dsv4_cuda_upload(const DSV4QMat *m);

/* include/dsv4/dsv4_cuda.h:83 -- 1 when m runs on the device: uploaded
 * itself, or a whole-row-block slice of an uploaded matrix. */
int dsv4_cuda_has(const DSV4QMat *m);

/* include/dsv4/dsv4_cuda.h:88 -- y[rows] = m * x[cols], host buffers,
 * synchronous. abort() if !dsv4_cuda_has(m), as the reference does. */
void dsv4_cuda_mmq(float *y, const float *x, const DSV4QMat *m);

/* include/dsv4/dsv4_cuda.h:94 -- x [nt][cols] -> y [nt][rows], one pass over
 * the weights per 8 tokens; nt <= DSV4_MAX_BATCH (abort otherwise). Each
 * token's result is bit-identical to a dsv4_cuda_mmq call. */
void dsv4_cuda_mmq_n(float *y, const float *x, const DSV4QMat *m, int nt);

/* include/dsv4/dsv4_cuda.h:97 -- bytes of HBM still free. */
size_t dsv4_cuda_free_vram(void);

/* include/dsv4/dsv4_cuda.h:99 -- release every device buffer. */
void dsv4_cuda_shutdown(void);

/* src/cuda/dsv4_cuda.cu:460 -- the device e4m3 decoder on all 256 codes. */
int dsv4_cuda_dump_e4m3(float *host256);

/* Release the device copy of an uploaded matrix (exact match only), so its
 * host buffer may be freed and its address reused. No reference counterpart:
 * the reference never releases a single matrix before shutdown. 0 or -1. */
int dsv4_cuda_evict(const DSV4QMat *m);

/* Device copies of a resident matrix (the slice's own rows for a slice), so
 * a caller can reach the same weights through the device API. 0 or -1. */
int dsv4_cuda_resident_ptrs(const DSV4QMat *m, const void **dw, const void **ds);

/* ---- MoE for one token: src/model/dsv4_layer.c:369-484 (moe) with the
 * router of src/core/dsv4_ops.c:102-141 (dsv4_route). ---- */
typedef struct dsv4b_moe dsv4b_moe;

/* Bind one layer's MoE to resident matrices. gate: router [n_experts][hidden]
 * (F32 / BF16 / FP8); bias: [n_experts] host floats or NULL (selection only,
 * as in the reference); experts: n_experts x {w1, w3, w2} descriptors, every
 * one uploaded (FP4 1x32 in the checkpoint); shared: {w1, w3, w2} or NULL,
 * added unweighted. score_func 1 = sqrt(softplus) (the reference's), 2 =
 * sigmoid. Returns NULL when a matrix is not resident or shapes disagree. */
dsv4b_moe *dsv4_cuda_moe_prepare(const DSV4QMat *gate, const float *bias,
                                 const DSV4QMat *experts, int n_experts,
                                 const DSV4QMat *shared, int topk,
                                 float route_scale, int score_func,
                                 float swiglu_limit);

/* out[hidden] = moe(x[hidden]) with host buffers, synchronous. fixed_experts
 * (topk ids) replaces top-k selection on hash-routed layers -- the caller's
 * tid2eid row, as dsv4_route takes it; NULL = score top-k. idx_out / w_out
 * (topk each, may be NULL) receive the routing decision. 0 or -1. */
int dsv4_cuda_moe(dsv4b_moe *m, float *out, const float *x,
                  const int *fixed_experts, int *idx_out, float *w_out);

void dsv4_cuda_moe_free(dsv4b_moe *m);

/* ---- sparse MLA, host buffers, synchronous ---- */

/* src/core/dsv4_indexer.c:64-85 -- out[n_pos] = indexer scores of the f32
 * key rows kv[n_pos][head_dim] for q[n_heads][head_dim] and the unscaled head
 * weights; the d^-1/2 * h^-1/2 scale is applied inside, as there. The
 * arithmetic is the reference's, so the scores are bit-identical. 0 or -1. */
int dsv4_cuda_indexer_score(float *out, const float *q, const float *kv,
                            const float *weights, int n_heads, int head_dim,
                            int n_pos);

/* src/core/dsv4_indexer.c:92-106 -- indices of the k largest scores,
 * descending, ties to the lower index, k clamped to n. Returns the count
 * written, or -1. */
int dsv4_cuda_topk(int *idxs, const float *scores, int n, int k);

/* src/core/dsv4_attn.c:60-108 -- o[h][d] = softmax attention of q[h][d] over
 * the rows of kv[.][d] named by idxs[topk] (-1 = masked), one shared KV head,
 * per-head sink in the denominator only. 0 or -1. */
int dsv4_cuda_sparse_attn(float *o, const float *q, const float *kv,
                          const float *sink, const int *idxs, int h, int d,
                          int topk, float scale);

/* ---- whole-token decode, every weight resident: the token loop of
 * src/cli/dsv4_run.c:444-483 around dsv4_layer_forward
 * (src/model/dsv4_layer.c:487-523), on the device. ---- */
typedef struct dsv4b_model dsv4b_model;

/* Copy a whole model to HBM: the structs the reference's binder fills
 * (dsv4_bind_layer / dsv4_bind_model), with the routed experts given as an
 * array experts[layer * n_experts + e] instead of the streaming cache. Host
 * memory is only read during the call. max_pos bounds the context (the
 * reference CLI uses sliding_window + 4096). NULL on failure. */
dsv4b_model *dsv4_cuda_model_create(const DSV4Cfg *c, const DSV4ModelW *mw,
                                    const DSV4LayerW *layers,
                                    const DSV4ExpertW *experts, int max_pos);

/* Start a sequence: empty caches, load the prompt, position 0. The first call
 * also captures one decode step into a CUDA graph. 0 or -1. */
int dsv4_cuda_model_begin(dsv4b_model *m, const int *prompt, int n_prompt);

/* Run the next position. *token receives the greedy argmax at it; logits
 * (vocab floats, may be NULL) its logits. The next position's input is the
 * prompt's token while prompt remains, else this argmax. 0 or -1. */
int dsv4_cuda_model_step(dsv4b_model *m, int *token, float *logits);

/* begin + n_prompt + n_gen steps; out receives the n_gen + 1 tokens emitted
 * from the last prompt position on. Returns that count, or -1. */
int dsv4_cuda_model_generate(dsv4b_model *m, const int *prompt, int n_prompt,
                             int n_gen, int *out);

/* One position driven by the host, the reference CLI's loop body
 * (dsv4_run.c:445-474): token at pos in, the greedy next token out.
 * Positions must follow each other from the last begin. 0 or -1. */
int dsv4_cuda_model_decode(dsv4b_model *m, int token, int pos, int *next_token);

/* A random-init model of configuration c generated directly in HBM (no host
 * weights): FP8 128x128 trunk from N(0, 0.02) (scales 2^-10), FP4 1x32
 * experts from N(0, 0.02) (scales 2^-6), BF16 router / compressor / indexer /
 * head N(0, 0.02), BF16 embedding N(0, 1), deterministic in seed. NULL if
 * it does not fit. */
dsv4b_model *dsv4_cuda_model_create_synthetic(const DSV4Cfg *c, int max_pos,
                                              unsigned long long seed);

/* ---- batched prefill (src/cli/dsv4_run.c:391-442, the --batch prompt
 * path; dsv4_layer_forward_n, src/model/dsv4_layer.c:856-918): the prompt
 * of a one-sequence model in passes of up to chunk tokens (1..64; the
 * reference's default is 32). Every launch of a pass covers all of its
 * tokens: mHC, every projection, the output projections, the MoE over the
 * union of the pass's experts, and the cache-bound core (q / KV finish,
 * compressor, indexer, top-k, attention). Each token still sees the window
 * and the compressor as they stood at its own position: the pass's KV rows
 * are staged beside the ring until the pass ends, and each compressor
 * window is pooled by the token that closes it. The head runs once, on the
 * prompt's last token.
 * Every token's arithmetic is that of a decode step, so the model is left
 * where dsv4_cuda_model_begin + n_prompt steps leave it: caches filled,
 * position n_prompt, the first generated token emitted. */

/* begin + the prompt in passes; returns the first generated token (the
 * argmax at position n_prompt - 1), or -1 (a batched or sharded model, or
 * chunk out of range). Steps and dsv4b_model_step_async continue from
 * position n_prompt. */
int dsv4b_model_prefill(dsv4b_model *m, const int *prompt, int n_prompt, int chunk);
/* dsv4_cuda_model_generate with the prompt prefilled in passes of chunk:
 * out receives the same n_gen + 1 tokens. Returns that count, or -1. */
int dsv4b_model_generate_prefill(dsv4b_model *m, const int *prompt, int n_prompt, int n_gen,
                                 int chunk, int *out);
/* The kernels the last prefill launched (each pass shape runs eagerly the
 * first time it is seen and as a captured graph after that), or -1 when a
 * pass of it ran eagerly. */
int dsv4b_model_prefill_kernels(const dsv4b_model *m);
/* The stream every call of the model enqueues on (a cudaStream_t): for
 * timing a synchronous call with events, or ordering other work after it. */
void *dsv4b_model_stream(const dsv4b_model *m);

/* ---- batched decode: n_seq sequences (<= 64) stepped in lockstep by one
 * graph. The reference's batched layer (dsv4_layer_forward_n,
 * src/model/dsv4_layer.c:856-918) runs nt tokens of ONE sequence and keeps
 * its attention strictly per token; here each of the n_seq sequences has its
 * own caches, prompt and greedy tokens, and every launch of the step covers
 * all of them (a grid dimension, or one GEMV item per sequence, so every
 * sequence's arithmetic is exactly that of a one-sequence model: its tokens
 * equal the ones dsv4_cuda_model_generate gives for its prompt). Needs the
 * fused mHC shapes (hc_mult <= 4) and one GPU. */
dsv4b_model *dsv4_cuda_model_create_batch(const DSV4Cfg *c, const DSV4ModelW *mw,
                                          const DSV4LayerW *layers,
                                          const DSV4ExpertW *experts, int max_pos, int n_seq);
dsv4b_model *dsv4_cuda_model_create_synthetic_batch(const DSV4Cfg *c, int max_pos,
                                                    unsigned long long seed, int n_seq);
int dsv4b_model_n_seq(const dsv4b_model *m);

/* dsv4_cuda_model_begin / _generate for a batch: prompts [n_seq][n_prompt]
 * (every prompt the same length); out [n_seq][n_gen + 1]. The
 * one-sequence calls (begin, step, generate, decode) return -1 on a batched
 * model; dsv4b_model_step_async steps every sequence. */
int dsv4b_model_begin_batch(dsv4b_model *m, const int *prompts, int n_prompt);
int dsv4b_model_generate_batch(dsv4b_model *m, const int *prompts, int n_prompt, int n_gen,
                               int *out);
/* dsv4_cuda_model_decode for a batch: tokens[n_seq] at position pos in,
 * next_tokens[n_seq] out. 0 or -1. */
int dsv4b_model_decode_batch(dsv4b_model *m, const int *tokens, int pos, int *next_tokens);

/* ---- multi-GPU decode (one process per GPU). No reference counterpart: the
 * reference runs on one device (dsv4_cuda.cu:243-249); this is the sharding
 * its design notes ask for -- routed and shared experts split along their
 * inter dimension on every rank, q heads (and with them wo_a's o_groups) by
 * rank, wo_b by the matching columns, the LM head by vocabulary -- with two
 * sums per layer over all ranks (the wo_b output, the experts' per-slot
 * outputs before the k-ordered combine) and one all-gather of the ranks'
 * argmax pairs per token. The sums run as one-shot exchanges over NVLink
 * peer memory by default (NCCL all-reduces with DSV4B_PEER=0); the argmax
 * gather is an NCCL all-gather. Every rank runs the same steps in lockstep. */

/* 0 if configuration c splits over world GPUs (heads, o_groups, wo_a / wo_b
 * 128-blocks, expert inter slices of whole 32-column FP4 scale blocks, the
 * shared expert's of 128 blocks, the vocabulary), else -1. No device needed. */
int dsv4b_shard_check(const DSV4Cfg *c, int world);

/* This rank's share of every split dimension as (first, count) pairs,
 * out[2 * k], out[2 * k + 1] for k = DSV4B_SHARD_HEADS .. DSV4B_SHARD_VOCAB:
 * q heads (and the sink), wq_b rows, o_groups, wo_a rows = wo_b columns (the
 * groups' o_lora slices), each routed expert's inter slice, the shared
 * expert's inter slice, LM-head rows. Ranks' shares tile each dimension in
 * rank order. Returns DSV4B_SHARD_NDIM, or -1 when c does not split over
 * world GPUs or rank is out of range. No device needed. */
enum {
    DSV4B_SHARD_HEADS = 0, DSV4B_SHARD_QROWS, DSV4B_SHARD_OGROUPS, DSV4B_SHARD_OLORA,
    DSV4B_SHARD_INTER, DSV4B_SHARD_SHARED_INTER, DSV4B_SHARD_VOCAB, DSV4B_SHARD_NDIM
};
int dsv4b_shard_plan(const DSV4Cfg *c, int world, int rank, int *out);

/* Size of the communicator id rank 0 creates and every rank passes to
 * dsv4_cuda_model_create_synthetic_sharded (NCCL's unique id, 128 bytes), and
 * its creation. NCCL is opened at run time; -1 when it cannot be. */
size_t dsv4b_nccl_id_bytes(void);
int dsv4b_nccl_unique_id(void *out);

/* This rank's share of the synthetic model of seed: every tensor is exactly
 * the corresponding slice of dsv4_cuda_model_create_synthetic's. Binds the
 * device first (dsv4_cuda_init, DSV4_DEVICE); nccl_id may be NULL for world 1.
 * NULL if c does not split over world or the model does not fit. */
dsv4b_model *dsv4_cuda_model_create_synthetic_sharded(const DSV4Cfg *c, int max_pos,
                                                      unsigned long long seed, int rank,
                                                      int world, const void *nccl_id);

/* The two per-layer sums run as one-shot exchanges over NVLink peer memory
 * (CUDA IPC mailboxes, one kernel each, every wait bounded) unless
 * DSV4B_PEER=0 selects NCCL all-reduces. 0 while every exchange has completed
 * in time; 1 once a wait for a rank gave up (the step's results are invalid);
 * -1 for a NULL model. Always 0 on one GPU. */
int dsv4b_model_comm_status(const dsv4b_model *m);

/* After a wait gave up, words a late rank still stores may sit in the
 * mailboxes: the model must be freed and created again before it exchanges
 * anything more. $DSV4B_PEER_SPIN sets the polls before a wait gives up
 * (default 2^26, a few seconds). No reference counterpart. */

/* Diagnostic: one peer exchange on ONE GPU with `world` ranks emulated in a
 * local mailbox. Ranks 1..world-1 have stored in[r*n .. r*n+n) beforehand
 * (others_ready) or never store (a rank that is gone, which the kernel must
 * survive by giving up after spin_limit polls); rank 0 contributes in[0..n)
 * and receives the rank-ordered sum in out[n]. Returns the status word (0 all
 * arrived, 1 a wait gave up) or -1. n a multiple of 4. No reference
 * counterpart. */
int dsv4b_peer_selftest(int world, int n, unsigned spin_limit, int others_ready,
                        const float *in, float *out);

/* Device memory in use (bytes), for reporting the resident model size. */
size_t dsv4_cuda_model_bytes(const dsv4b_model *m);

/* Kernel launches in one decode step: the kernel nodes of the captured step
 * graph (copies excluded). -1 before the first dsv4_cuda_model_begin. */
int dsv4_cuda_model_step_kernels(const dsv4b_model *m);

void dsv4_cuda_model_free(dsv4b_model *m);

/* ===================================================== 2. device API ====== */

/* y[t*rows + o] = sum_c W[o][c] * x[t*cols + c] for t < nt; any nt >= 1.
 * W/S are device pointers in the storage format `wdt`. 0 or -1. */
int dsv4b_gemv(int wdt, float *y, const float *x, const void *W, const void *S,
               int rows, int cols, int blk_r, int blk_c, int nt, void *stream);

/* Element types of key / KV rows in the sparse-MLA device entries. */
enum { DSV4B_F32 = 0, DSV4B_BF16 = 1, DSV4B_E4M3 = 2 };

/* Indexer scores for `batch` sequences: out[b][t], t < n_pos, from
 * q[b][n_heads][head_dim], head weights w[b][n_heads] and key rows of type
 * key_dt at keys + b*seq_key_stride + t*key_stride (elements). `scale` is the
 * reference's d^-1/2 * h^-1/2 (the caller computes it in float). */
int dsv4b_indexer_score(float *out, const float *q, const void *keys,
                        int key_dt, long key_stride, long seq_key_stride,
                        const float *w, int n_heads, int head_dim, int n_pos,
                        float scale, int batch, void *stream);

/* Top-k per sequence: idx[b][min(k,n)] of scores[b][n]. n <= 47104, k <= 4096. */
int dsv4b_topk(int *idx, const float *scores, int n, int k, int batch,
               void *stream);

/* Sparse attention per sequence: o[b][n_heads][d] over the KV rows
 * (type kv_dt, seq_kv_rows rows of width d per sequence) named by
 * idxs[b][topk]. `scratch` holds dsv4b_sparse_attn_scratch() bytes. */
size_t dsv4b_sparse_attn_scratch(int n_heads, int d, int topk, int batch);
int dsv4b_sparse_attn(float *o, const float *q, const void *kv, int kv_dt,
                      long seq_kv_rows, const float *sink, const int *idxs,
                      int n_heads, int d, int topk, float scale, int batch,
                      void *scratch, size_t scratch_bytes, void *stream);

/* dsv4b_sparse_attn with its scratch in a fixed 8 MiB device array instead
 * of caller memory: no call allocates. No reference counterpart (the
 * reference's attention runs on the host); it is for callers with no device
 * allocator of their own or no HBM left to give. The first call on a device
 * sets up (looks up the array's address) and should come before any stream
 * capture; calls in flight at the same time on one device race on the one
 * array. Returns 0, -1 on a bad argument or CUDA error, -2 when
 * dsv4b_sparse_attn_scratch(n_heads, d, topk, batch) exceeds
 * DSV4B_SPARSE_ATTN_STATIC_SCRATCH. */
#define DSV4B_SPARSE_ATTN_STATIC_SCRATCH ((size_t)8 << 20)
int dsv4b_sparse_attn_static(float *o, const float *q, const void *kv, int kv_dt,
                             long seq_kv_rows, const float *sink, const int *idxs,
                             int n_heads, int d, int topk, float scale, int batch,
                             void *stream);

/* The prepared MoE on device buffers x[hidden] -> out[hidden], stream-ordered. */
int dsv4b_moe_forward(dsv4b_moe *m, float *out, const float *x, void *stream);

/* Enqueue one decode step (the captured graph) on `stream` without waiting;
 * dsv4_cuda_model_begin must have run. 0 or -1. */
int dsv4b_model_step_async(dsv4b_model *m, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* DSV4_B200_H */

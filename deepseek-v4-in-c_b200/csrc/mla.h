// mla.h - sparse MLA decode kernels (mla.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#define DSV4B_DT_F32 0
#define DSV4B_DT_BF16 1
#define DSV4B_DT_E4M3 2

namespace dsv4b {

constexpr int kTopkMaxN = 49152;    // scores held in shared memory
constexpr int kTopkMaxK = 4096;
constexpr int kTopkEqCap = 1024;    // ties at the k-th score ranked directly (more: an ordered scan)

// out[b][t] for t < n_pos: the reference's indexer score of key row t.
// keys of sequence b start at keys + b*seq_key_stride elements; row t at
// t*key_stride elements; q is [batch][n_heads][head_dim], w [batch][n_heads].
int indexer_score(float *out, const float *q, const void *keys, int key_dt, long key_stride,
                  long seq_key_stride, const float *w, int n_heads, int head_dim, int n_pos,
                  float scale, int batch, cudaStream_t st, const int *dyn_n = nullptr,
                  double *terms = nullptr, unsigned *count = nullptr, int dyn_stride = 0);
// terms / count (optional, both or neither): scratch for the head-split
// form, [batch][n_pos][n_heads] doubles and [batch][ceil(n_pos / 32)]
// counters that start (and are left) at zero; same results.
// dyn_n (device, may be null): the rows that exist, <= n_pos; one count for
// every sequence, or with dyn_stride sequence b's at dyn_n[b * dyn_stride].
// idx[b][i], i < min(k, n): descending scores, ties to the lower index.
// dyn_nk (device, may be null): {n, k} of this step, n <= the launch's n and
// k <= the launch's k (the launch sizes shared memory for the maxima); with
// dyn_stride, sequence b's pair at dyn_nk + b * dyn_stride.
int topk(int *idx, const float *scores, int n, int k, int batch, long seq_in_stride,
         long seq_out_stride, cudaStream_t st, const int *dyn_nk = nullptr, int dyn_stride = 0);
size_t attn_part_bytes(int n_heads, int d, int topk, int batch);
// o[b][h][d]; kv of sequence b is rows [b*seq_kv_rows, ...) of width d; idxs
// [b][topk] with -1 = masked; part_buf holds attn_part_bytes().
// Optional de-rotation of every output head (inverse RoPE of its last rd
// dims at table row pos[b * pos_stride] for sequence b), done by the kernel
// that writes the head.
struct AttnRope {
    const float *cs, *sn;
    const int *pos;
    int rd;
    int pos_stride;
};
int sparse_attn(float *o, const float *q, const void *kv, int kv_dt, long seq_kv_rows,
                const float *sink, const int *idxs, long seq_idx_stride, int n_heads, int d,
                int topk, float scale, int batch, void *part_buf, cudaStream_t st,
                const AttnRope *rope = nullptr);

}  // namespace dsv4b

// capi_mla.cu - C ABI of the sparse-MLA kernels: host-buffer twins of the
// reference's dsv4_indexer_score / dsv4_topk / dsv4_sparse_attn (same
// arguments and meaning) and the batched device entries.
#include <stdlib.h>
#include <string.h>

#include "common.cuh"
#include "internal.h"
#include "mla.h"
#include "../../include/dsv4_b200.h"

using namespace dsv4b;

namespace {

// Grow-only device buffers for the host-buffer entries.
struct HostScratch {
    void *p = nullptr;
    size_t cap = 0;
    void *get(size_t n)
    {
        if (n > cap) {
            if (p) cudaFree(p);
            p = nullptr;
            cap = 0;
            if (cudaMalloc(&p, n) != cudaSuccess) return nullptr;
            cap = n;
        }
        return p;
    }
};
HostScratch hs_a, hs_b, hs_c, hs_d, hs_e;

// The host-buffer entries bring the device up on first use, as
// dsv4_cuda_dump_e4m3 does.
bool ready()
{
    return dsv4_cuda_init() == 0;
}

}  // namespace

extern "C" int dsv4_cuda_indexer_score(float *out, const float *q, const float *kv, const float *weights,
                                       int n_heads, int head_dim, int n_pos)
{
    if (n_pos <= 0) return 0;
    if (!out || !q || !kv || !weights || n_heads <= 0 || head_dim <= 0 || !ready()) return -1;
    const size_t qb = (size_t)n_heads * head_dim * 4, kb = (size_t)n_pos * head_dim * 4;
    float *dq = (float *)hs_a.get(qb), *dk = (float *)hs_b.get(kb), *dw = (float *)hs_c.get(n_heads * 4);
    float *dout = (float *)hs_d.get((size_t)n_pos * 4);
    if (!dq || !dk || !dw || !dout) return -1;
    cudaStream_t st = stream_of(nullptr);
    DSV4B_CUDA_OK(cudaMemcpyAsync(dq, q, qb, cudaMemcpyHostToDevice, st));
    DSV4B_CUDA_OK(cudaMemcpyAsync(dk, kv, kb, cudaMemcpyHostToDevice, st));
    DSV4B_CUDA_OK(cudaMemcpyAsync(dw, weights, n_heads * 4, cudaMemcpyHostToDevice, st));
    // the reference's scale: (1/sqrtf(head_dim)) * (1/sqrtf(n_heads)) in float
    const float scale = (1.0f / sqrtf((float)head_dim)) * (1.0f / sqrtf((float)n_heads));
    if (indexer_score(dout, dq, dk, DSV4B_DT_F32, head_dim, 0, dw, n_heads, head_dim, n_pos, scale, 1, st))
        return -1;
    DSV4B_CUDA_OK(cudaMemcpyAsync(out, dout, (size_t)n_pos * 4, cudaMemcpyDeviceToHost, st));
    DSV4B_CUDA_OK(cudaStreamSynchronize(st));
    return 0;
}

extern "C" int dsv4_cuda_topk(int *idxs, const float *scores, int n, int k)
{
    if (k > n) k = n;
    if (k <= 0) return 0;
    if (!idxs || !scores || !ready()) return -1;
    float *ds = (float *)hs_a.get((size_t)n * 4);
    int *di = (int *)hs_b.get((size_t)k * 4);
    if (!ds || !di) return -1;
    cudaStream_t st = stream_of(nullptr);
    DSV4B_CUDA_OK(cudaMemcpyAsync(ds, scores, (size_t)n * 4, cudaMemcpyHostToDevice, st));
    if (topk(di, ds, n, k, 1, n, k, st)) return -1;
    DSV4B_CUDA_OK(cudaMemcpyAsync(idxs, di, (size_t)k * 4, cudaMemcpyDeviceToHost, st));
    DSV4B_CUDA_OK(cudaStreamSynchronize(st));
    return k;
}

extern "C" int dsv4_cuda_sparse_attn(float *o, const float *q, const float *kv, const float *sink,
                                     const int *idxs, int h, int d, int topk_n, float scale)
{
    if (!o || !q || !kv || !sink || !idxs || h <= 0 || d <= 0 || topk_n < 0 || !ready()) return -1;
    int nrows = 0;
    for (int j = 0; j < topk_n; j++) nrows = idxs[j] + 1 > nrows ? idxs[j] + 1 : nrows;
    const size_t qb = (size_t)h * d * 4, kb = (size_t)(nrows > 0 ? nrows : 1) * d * 4;
    float *dq = (float *)hs_a.get(qb), *dk = (float *)hs_b.get(kb), *dsk = (float *)hs_c.get((size_t)h * 4);
    int *di = (int *)hs_d.get((size_t)(topk_n > 0 ? topk_n : 1) * 4);
    float *dout = (float *)hs_e.get(qb + attn_part_bytes(h, d, topk_n > 0 ? topk_n : 1, 1));
    if (!dq || !dk || !dsk || !di || !dout) return -1;
    cudaStream_t st = stream_of(nullptr);
    if (topk_n == 0) {
        memset(o, 0, qb);
        return 0;
    }
    DSV4B_CUDA_OK(cudaMemcpyAsync(dq, q, qb, cudaMemcpyHostToDevice, st));
    if (nrows > 0) DSV4B_CUDA_OK(cudaMemcpyAsync(dk, kv, (size_t)nrows * d * 4, cudaMemcpyHostToDevice, st));
    DSV4B_CUDA_OK(cudaMemcpyAsync(dsk, sink, (size_t)h * 4, cudaMemcpyHostToDevice, st));
    DSV4B_CUDA_OK(cudaMemcpyAsync(di, idxs, (size_t)topk_n * 4, cudaMemcpyHostToDevice, st));
    if (sparse_attn(dout, dq, dk, DSV4B_DT_F32, nrows, dsk, di, topk_n, h, d, topk_n, scale, 1,
                    (char *)dout + qb, st))
        return -1;
    DSV4B_CUDA_OK(cudaMemcpyAsync(o, dout, qb, cudaMemcpyDeviceToHost, st));
    DSV4B_CUDA_OK(cudaStreamSynchronize(st));
    return 0;
}

extern "C" int dsv4b_indexer_score(float *out, const float *q, const void *keys, int key_dt, long key_stride,
                                   long seq_key_stride, const float *w, int n_heads, int head_dim, int n_pos,
                                   float scale, int batch, void *stream)
{
    if (key_dt < 0 || key_dt > 2) return -1;
    return indexer_score(out, q, keys, key_dt, key_stride, seq_key_stride, w, n_heads, head_dim, n_pos, scale,
                         batch, stream_of(stream));
}

extern "C" int dsv4b_topk(int *idx, const float *scores, int n, int k, int batch, void *stream)
{
    const int kk = k < n ? k : n;
    return topk(idx, scores, n, k, batch, n, kk, stream_of(stream));
}

extern "C" size_t dsv4b_sparse_attn_scratch(int n_heads, int d, int topk_n, int batch)
{
    return attn_part_bytes(n_heads, d, topk_n, batch);
}

extern "C" int dsv4b_sparse_attn(float *o, const float *q, const void *kv, int kv_dt, long seq_kv_rows,
                                 const float *sink, const int *idxs, int n_heads, int d, int topk_n,
                                 float scale, int batch, void *scratch, size_t scratch_bytes, void *stream)
{
    if (kv_dt < 0 || kv_dt > 2 || !scratch) return -1;
    if (scratch_bytes < attn_part_bytes(n_heads, d, topk_n, batch)) return -1;
    return sparse_attn(o, q, kv, kv_dt, seq_kv_rows, sink, idxs, topk_n, n_heads, d, topk_n, scale, batch,
                       scratch, stream_of(stream));
}

// capi_static.cu - sparse attention whose scratch lives in a fixed device
// array, so a call allocates no memory.
//
// dsv4b_sparse_attn needs dsv4b_sparse_attn_scratch() bytes of device memory
// for its per-chunk partials. Some callers cannot provide that: a caller that
// reaches the kernels through a plain C loop with no device allocator of its
// own (the reference's layer code holds only host arrays), or a caller whose
// HBM is entirely carved up for resident weights and KV caches at start-up.
// Such a caller also cannot let the call allocate on its behalf, because
// cudaMalloc / cudaFree synchronise the whole device and would stall every
// other stream in the decode loop. This entry point keeps the partials in
// kStaticScratch bytes of statically sized device memory instead, reserved
// when the module is loaded.
//
// Rules for callers:
//   * the first call on each device looks up the array's device address with
//     that device current (cudaGetSymbolAddress); make that first call before
//     any stream capture is begun;
//   * the partials are written in full by every call before they are read,
//     so nothing in the array has to start at zero;
//   * there is one array per device: two calls in flight at the same time on
//     one device (different streams, or different host threads without
//     ordering between their streams) race on it and both results are
//     undefined. Issue them on one stream, or order them.
#include <mutex>
#include <stdio.h>

#include "internal.h"
#include "mla.h"
#include "../../include/dsv4_b200.h"

namespace dsv4b {
namespace {

constexpr size_t kStaticScratch = DSV4B_SPARSE_ATTN_STATIC_SCRATCH;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_attn_scratch[kStaticScratch];

std::mutex g_mu;
void *g_ptr[kMaxDevices];  // device address of g_attn_scratch per device

// Device address of this device's copy of the array, looked up once.
void *scratch_for_current_device()
{
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_ptr[dev]) {
        void *p = nullptr;
        const cudaError_t rc = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (rc != cudaSuccess) {
            fprintf(stderr, "dsv4b_sparse_attn_static: cudaGetSymbolAddress failed on device %d: %s\n", dev,
                    cudaGetErrorString(rc));
            return nullptr;
        }
        g_ptr[dev] = p;
    }
    return g_ptr[dev];
}

}  // namespace
}  // namespace dsv4b

using namespace dsv4b;

extern "C" int dsv4b_sparse_attn_static(float *o, const float *q, const void *kv, int kv_dt, long seq_kv_rows,
                                        const float *sink, const int *idxs, int n_heads, int d, int topk_n,
                                        float scale, int batch, void *stream)
{
    if (kv_dt < 0 || kv_dt > 2) return -1;
    if (batch <= 0 || topk_n <= 0) return 0;
    // the shapes sparse_attn accepts, checked before the scratch size is
    // computed from them (a negative count would wrap it)
    if (n_heads <= 0 || d <= 0 || d > 1024 || (d & 3)) return -1;
    const size_t need = attn_part_bytes(n_heads, d, topk_n, batch);
    if (need > kStaticScratch) {
        fprintf(stderr,
                "dsv4b_sparse_attn_static: heads=%d d=%d topk=%d batch=%d needs %zu bytes of scratch, "
                "above the fixed %zu; use dsv4b_sparse_attn with caller scratch\n",
                n_heads, d, topk_n, batch, need, kStaticScratch);
        return -2;
    }
    void *scratch = scratch_for_current_device();
    if (!scratch) return -1;
    return sparse_attn(o, q, kv, kv_dt, seq_kv_rows, sink, idxs, topk_n, n_heads, d, topk_n, scale, batch,
                       scratch, stream_of(stream));
}

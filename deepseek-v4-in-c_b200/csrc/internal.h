// internal.h - declarations shared between the backend's translation units.
// Not part of the public C ABI (that is include/dsv4_b200.h).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace dsv4b {

constexpr int kGemvMaxItems = 16;

// One matrix of a grouped batch-1 GEMV launch: y[rows] = W x, or with pair
// set, y = SwiGLU(W x, W2 x) with the reference's clamp at `limit`. Routed
// experts are picked on the device: with wtab set, W = wtab[sel[slot]] and
// S = stab[sel[slot]] (W2 / S2 from w2tab / s2tab).
struct GemvItem {
    const uint8_t *W, *S, *W2, *S2;
    const uint8_t *const *wtab, *const *stab, *const *w2tab, *const *s2tab;
    const int *sel;
    const float *x;
    float *y;
    int fmt, rows, cols, sc, lbr, lbc, rowbytes, slot, pair;
    int mma;                // on the tensor cores (gemv_mma.cuh)
    // Routed items of a batch (tensor-core items only): with perm set, the
    // item is group `slot` of a device-side list (perm[5 slot] tokens, 0 for
    // an unused slot, entries (token << 8) | k at perm[5 slot + 1 ..]): for
    // each entry it reads x + token xs + k xk and writes y + token ys + k yk;
    // the group's expert is sel[token ss + k] of its first entry. Every
    // token's arithmetic is that of a single-token item.
    const int *perm;
    int xs, xk, ys, yk, ss;
    // Tokens of one item (tensor-core items): nt > 1 applies the matrix to nt
    // vectors x + i xts with results at y + i yts, streaming it once.
    int nt, xts, yts;
    float limit;
    int tile0, tr;          // first block of this item; virtual rows per block
};

struct GemvBatch {
    GemvItem it[kGemvMaxItems];
    int n;
};

size_t row_bytes(int fmt, int cols);
// Whether a matrix takes the tensor-core path: FP8 (column blocks of 128 or
// more) or BF16 in whole 128-column units, FP4 (1x32 blocks) in whole
// 256-column units whose scales all lie in 2^-23..2^1 (f16s: the holder of
// the scales has checked), at most 64 units per row. A function of the
// matrix only, so one matrix always sums in one order, whatever the batch.
bool gemv_mma_shape(int fmt, int cols, int blk_r, int blk_c, bool f16s);
// Whether every E8M0 scale byte lets an e2m1 value times the scale be an
// exact f16 through the tensor-core decode (exponents -23..1).
bool fp4_scales_f16(const uint8_t *s, size_t n);
// An item for W (or the table triple, when W is null) of the given shape;
// false when the shape cannot take the 128-bit streaming kernels (rows not a
// multiple of 16 bytes, unaligned pointers, scale blocks not powers of two
// of at least 4 columns).
bool gemv_item(GemvItem &it, int fmt, const void *W, const uint8_t *S, int rows, int cols, int blk_r,
               int blk_c, const float *x, float *y, bool f16s = false);
// One launch over n <= kGemvMaxItems items (blocks planned here).
int gemv_group(GemvItem *items, int n, cudaStream_t st);
// Give a tensor-core item up to `want` tokens (x / y xts / yts floats apart),
// as many as its shared memory allows; returns the tokens it now covers (1
// for other items, which stay single-token).
int gemv_item_tokens(GemvItem &it, int want, long xts, long yts);
bool gemv_vectorizable(int fmt, const void *W, int cols, int blk_r, int blk_c, const float *x, long xstride);
// y[t*ystride + o] = sum_c W[o][c] * x[t*xstride + c], t < nt, o < rows.
int gemv(int fmt, float *y, long ystride, const float *x, long xstride, const void *W, const uint8_t *S,
         int rows, int cols, int blk_r, int blk_c, int nt, cudaStream_t st, bool f16s = false);
int dump_e4m3(float *dev_out, cudaStream_t st);

// Multi-GPU exchange (comm.cu): NCCL opened at run time. comm is an NCCL
// communicator or null (one GPU: every call is a no-op returning 0).
size_t comm_id_bytes();
int comm_unique_id(void *out);
int comm_open(void **comm, int rank, int world, const void *id);
void comm_close(void *comm);
int comm_allreduce_sum(float *buf, size_t n, void *comm, cudaStream_t st);
int comm_allgather(const void *send, void *recv, size_t bytes_per_rank, void *comm, cudaStream_t st);
// One-shot sum all-reduce over NVLink peer memory (CUDA IPC mailboxes, one
// kernel, bounded waits): opened once per model over an NCCL communicator;
// n <= maxn floats, a multiple of 4; exchange `call` of a step of nx
// exchanges, the step count at *stepseq. peer_status: 0, or 1 once a wait
// timed out.
int peer_open(void **peer, int rank, int world, int maxn, void *comm, cudaStream_t st);
void peer_close(void *peer);
int peer_allreduce_sum(void *peer, float *buf, int n, const unsigned *stepseq, int nx, int call, cudaStream_t st);
int peer_status(void *peer);
// Where a sharded step's sums go: the peer exchange when open, else NCCL (or
// nothing on one GPU). *call counts the step's exchanges as they are enqueued.
struct Exch {
    void *peer, *comm;
    const unsigned *stepseq;
    int nx;
    int *call;
};
int xreduce_sum(const Exch &x, float *buf, size_t n, cudaStream_t st);

// The backend's own stream (NULL stream arguments of the device API).
cudaStream_t stream_of(void *s);

// Raises kernel's dynamic shared memory limit to `bytes` on the CURRENT
// device. The attribute belongs to each device's context, so it is set once
// per (device, kernel) -- under a lock, any host thread -- and its return code
// is checked; 0 or -1.
int smem_optin(const void *kernel, int bytes);
template <typename... A>
static inline int smem_optin(void (*kernel)(A...), int bytes)
{
    return smem_optin(reinterpret_cast<const void *>(kernel), bytes);
}

// Whether kernels are launched as programmatic dependents of their
// predecessor ($DSV4B_PDL=0 turns it off).
bool pdl_enabled();

// Programmatic dependent launch is used only inside kernel chains this
// backend enqueues itself (a decode step, an MoE forward): the first launch
// of a chain is ordinary -- its predecessor may be a copy, which
// griddepcontrol.wait does not wait for, or a caller's kernel -- and every
// later launch of the chain may overlap the kernel before it. Chains nest.
extern thread_local int t_chain;    // depth of chains being enqueued
extern thread_local bool t_pdl;     // the next launch follows a kernel of this chain
struct PdlChain {
    PdlChain()
    {
        if (t_chain++ == 0) t_pdl = false;
    }
    ~PdlChain()
    {
        if (--t_chain == 0) t_pdl = false;
    }
};

// kernel<<<grid, block, smem, st>>>(args...), as a programmatic dependent of
// the previous kernel when inside a chain; every kernel launched this way
// starts with pdl_trigger() and calls pdl_wait() before touching its
// predecessor's data.
template <typename... KArgs, typename... Args>
static inline cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                 cudaStream_t st, Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = (t_chain > 0 && t_pdl && pdl_enabled()) ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, (KArgs)args...);
    if (t_chain > 0) t_pdl = true;
    return e;
}

}  // namespace dsv4b

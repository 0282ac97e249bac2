// internal.h - declarations shared between the backend's translation units.
// Not part of the public C ABI (that is include/dsv4_b200.h).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace dsv4b {

struct GemvArgs {
    float *y;
    const float *x;
    const uint8_t *W;
    const uint8_t *S;
    int rows, cols, blk_r, blk_c, sc, rowbytes;
    int lbr, lbc;           // log2 of the (power-of-two) block sizes
    long xstride, ystride;
    // Device-side matrix selection (routed experts): when wtab != nullptr the
    // weights are wtab[sel[slot]] and the scales stab[sel[slot]].
    const uint8_t *const *wtab;
    const uint8_t *const *stab;
    const int *sel;
    int slot;
};

// One matrix of a grouped TMA GEMV launch. With sel >= 0 the weights are
// W + sel_idx[sel] * wstride (and S likewise): a routed expert picked on the
// device, read without a host round trip.
struct TmaGroup {
    const uint8_t *W, *S;
    long wstride, sstride;
    const float *x;
    float *y;
    int rows, sel;
};

constexpr int kTmaMaxGroups = 16;

size_t row_bytes(int fmt, int cols);
bool gemv_vectorizable(int fmt, const void *W, int cols, int blk_r, int blk_c,
                       const float *x, long xstride);
// y[t*ystride + o] = sum_c W[o][c] * x[t*xstride + c], t < nt, o < rows.
int gemv(int fmt, float *y, long ystride, const float *x, long xstride,
         const void *W, const uint8_t *S, int rows, int cols, int blk_r,
         int blk_c, int nt, cudaStream_t st);
int gemv_reg(const GemvArgs &g, int fmt, int nt, cudaStream_t st);
// Batch-1 GEMV whose weights are picked on the device: W = wtab[sel[slot]].
int gemv_sel(int fmt, float *y, const float *x, const uint8_t *const *wtab,
             const uint8_t *const *stab, const int *sel, int slot, int rows,
             int cols, int blk_r, int blk_c, cudaStream_t st);
bool gemv_tma_ok(int fmt, const GemvArgs &g);
// Batch-1 GEMV of up to kTmaMaxGroups matrices sharing format and width.
int gemv_tma(int fmt, const TmaGroup *grp, int ngroups, int cols, int blk_r,
             int blk_c, const int *sel_idx, cudaStream_t st);
int dump_e4m3(float *dev_out, cudaStream_t st);

// Per-device scratch of the split-tile protocol (segment partial sums and
// arrival counters), allocated once at init. Counters return to zero at the
// end of every launch.
struct Workspace {
    float *segbuf;
    int *cnt;
    int *err;
    int slots;
    int nsm;
};
Workspace &workspace();
// The backend's own stream (NULL stream arguments of the device API).
cudaStream_t stream_of(void *s);
int workspace_init();
void workspace_free();

}  // namespace dsv4b

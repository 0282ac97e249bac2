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
    float limit;
    int tile0, tr;          // first block of this item; virtual rows per block
};

struct GemvBatch {
    GemvItem it[kGemvMaxItems];
    int n;
};

size_t row_bytes(int fmt, int cols);
// An item for W (or the table triple, when W is null) of the given shape;
// false when the shape cannot take the 128-bit streaming kernels (rows not a
// multiple of 16 bytes, unaligned pointers, scale blocks not powers of two
// of at least 4 columns).
bool gemv_item(GemvItem &it, int fmt, const void *W, const uint8_t *S, int rows, int cols, int blk_r,
               int blk_c, const float *x, float *y);
// One launch over n <= kGemvMaxItems items (blocks planned here).
int gemv_group(GemvItem *items, int n, cudaStream_t st);
bool gemv_vectorizable(int fmt, const void *W, int cols, int blk_r, int blk_c, const float *x, long xstride);
// y[t*ystride + o] = sum_c W[o][c] * x[t*xstride + c], t < nt, o < rows.
int gemv(int fmt, float *y, long ystride, const float *x, long xstride, const void *W, const uint8_t *S,
         int rows, int cols, int blk_r, int blk_c, int nt, cudaStream_t st);
int dump_e4m3(float *dev_out, cudaStream_t st);

// The backend's own stream (NULL stream arguments of the device API).
cudaStream_t stream_of(void *s);

}  // namespace dsv4b

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
    long xstride, ystride;
};

size_t row_bytes(int fmt, int cols);
bool gemv_vectorizable(int fmt, const void *W, int cols, int blk_c,
                       const float *x, long xstride);
// y[t*ystride + o] = sum_c W[o][c] * x[t*xstride + c], t < nt, o < rows.
int gemv(int fmt, float *y, long ystride, const float *x, long xstride,
         const void *W, const uint8_t *S, int rows, int cols, int blk_r,
         int blk_c, int nt, cudaStream_t st);
int dump_e4m3(float *dev_out, cudaStream_t st);

}  // namespace dsv4b

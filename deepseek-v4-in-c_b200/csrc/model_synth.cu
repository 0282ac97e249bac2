// model_synth.cu - a random-init model generated directly in HBM.
//
// BASELINE config 5 is ~156 GB of weights: too much to build on the host and
// copy. This fills every tensor on the device from a counter-based hash of
// (seed, tensor, index), so the model is deterministic in the seed:
//   FP8 128x128 trunk  codes = e4m3(N(0,1) * 0.02 / 2^-10), block scales 2^-10
//                      (config 1: at sigma 0.02 every block's absmax/448 rounds
//                      up below 2^-10, so every block clamps to 2^-10);
//   FP4 1x32 experts   codes = e2m1(N(0,1) * 0.02 / 2^-6), scales 2^-6 (the
//                      power of two 2^ceil(log2(absmax/6)) of 32 N(0, 0.02)
//                      draws);
//   BF16               N(0, 0.02) (router, compressor, indexer weights, head),
//                      N(0, 1) for the embedding;
//   f32                norms 1 + 0.1 N, mHC fn 0.02 N, base 0.5 N, scale in
//                      [0.5, 1), sinks N(0, 1), compressor ape 0.1 N, router
//                      bias 0.05 N; tid2eid rows of distinct experts.
// The rounding to e4m3 / e2m1 uses the hardware converters (round to nearest
// even, saturating).
#include <math.h>

#include <vector>

#include "common.cuh"
#include "internal.h"
#include "model.h"
#include "../../include/dsv4_b200.h"

namespace dsv4b {

__device__ __forceinline__ uint64_t mix64(uint64_t z)
{
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Standard normal number i of stream `key` (Box-Muller on two 24-bit uniforms).
__device__ __forceinline__ float nrand(uint64_t key, uint64_t i)
{
    const uint64_t h = mix64(key ^ mix64(i));
    const float u1 = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = (float)((h >> 16) & 0xFFFFFFu) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

__device__ __forceinline__ float urand(uint64_t key, uint64_t i)
{
    return (float)(mix64(key ^ mix64(i)) >> 40) * (1.0f / 16777216.0f);
}

// kind: 0 f32 a + b*N, 1 f32 a + b*U, 2 bf16 b*N, 3 e4m3 codes of b*N, 4 e2m1
// packed codes of b*N, 5 constant byte a
__global__ void k_synth(void *dst, size_t n, int kind, float a, float b, uint64_t key)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        switch (kind) {
        case 0: reinterpret_cast<float *>(dst)[i] = a + b * nrand(key, i); break;
        case 1: reinterpret_cast<float *>(dst)[i] = a + b * urand(key, i); break;
        case 2: {
            const float v = b * nrand(key, i);
            reinterpret_cast<uint16_t *>(dst)[i] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
            break;
        }
        case 3: {
            const float v = b * nrand(key, i);
            reinterpret_cast<uint8_t *>(dst)[i] = (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
            break;
        }
        case 4: {  // byte i holds elements 2i (low nibble) and 2i+1
            const float2 v = make_float2(b * nrand(key, 2 * i), b * nrand(key, 2 * i + 1));
            reinterpret_cast<uint8_t *>(dst)[i] = (uint8_t)__nv_cvt_float2_to_fp4x2(v, __NV_E2M1, cudaRoundNearest);
            break;
        }
        default: reinterpret_cast<uint8_t *>(dst)[i] = (uint8_t)a; break;
        }
    }
}

// A slice of a synthetic tensor, identical to the same elements of the whole
// one: element (i, j) of the [nrows][ncols] slice is element
// base + i * gstride + j of the tensor's stream (kinds 0..3 and 5 of k_synth).
__global__ void k_synth_slice(void *dst, int nrows, int ncols, int kind, float a, float b, uint64_t key,
                              size_t base, size_t gstride)
{
    const size_t n = (size_t)nrows * ncols;
    for (size_t li = blockIdx.x * (size_t)blockDim.x + threadIdx.x; li < n; li += (size_t)gridDim.x * blockDim.x) {
        const size_t i = li / ncols, j = li - i * ncols, gi = base + i * gstride + j;
        switch (kind) {
        case 0: reinterpret_cast<float *>(dst)[li] = a + b * nrand(key, gi); break;
        case 1: reinterpret_cast<float *>(dst)[li] = a + b * urand(key, gi); break;
        case 2: {
            const float v = b * nrand(key, gi);
            reinterpret_cast<uint16_t *>(dst)[li] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
            break;
        }
        case 3: {
            const float v = b * nrand(key, gi);
            reinterpret_cast<uint8_t *>(dst)[li] = (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
            break;
        }
        default: reinterpret_cast<uint8_t *>(dst)[li] = (uint8_t)a; break;
        }
    }
}

// The routed experts' e2m1 codes of one layer for one rank's inter slice
// [i0, i0 + il) (i0 even): the whole layer is one stream of packed bytes,
// expert e at e * cper, its w1, w3 ([inter][hidden / 2] bytes) and w2
// ([hidden][inter / 2]) one after the other. A rank keeps rows [i0, i0 + il)
// of w1 and w3 and the same columns of w2, stored as one compact block per
// expert: [w1 slice][w3 slice][w2 slice].
__global__ void k_synth_experts(uint8_t *dst, int n_experts, int hidden, int inter, int i0, int il_, float b,
                                uint64_t key)
{
    const size_t il = il_, cw = (size_t)inter * hidden / 2, cper = 3 * cw;
    const size_t cwl = il * hidden / 2, cperl = 3 * cwl, n = (size_t)n_experts * cperl;
    const size_t w2rb = inter / 2, w2rbl = il / 2;
    for (size_t lb = blockIdx.x * (size_t)blockDim.x + threadIdx.x; lb < n; lb += (size_t)gridDim.x * blockDim.x) {
        const size_t e = lb / cperl, rem = lb - e * cperl;
        size_t gb;
        if (rem < 2 * cwl) {
            const size_t jm = rem / cwl, off = rem - jm * cwl, row = off / (hidden / 2), cb = off - row * (hidden / 2);
            gb = e * cper + jm * cw + (i0 + row) * (hidden / 2) + cb;
        } else {
            const size_t off = rem - 2 * cwl, row = off / w2rbl, cb = off - row * w2rbl;
            gb = e * cper + 2 * cw + row * w2rb + i0 / 2 + cb;
        }
        const float2 v = make_float2(b * nrand(key, 2 * gb), b * nrand(key, 2 * gb + 1));
        dst[lb] = (uint8_t)__nv_cvt_float2_to_fp4x2(v, __NV_E2M1, cudaRoundNearest);
    }
}

__global__ void k_synth_tid2eid(int64_t *t, int vocab, int topk, int n_experts, uint64_t key)
{
    for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < vocab; v += gridDim.x * blockDim.x) {
        const int base = (int)(mix64(key ^ (uint64_t)v) % (uint64_t)n_experts);
        for (int k = 0; k < topk; k++) t[(size_t)v * topk + k] = (base + k) % n_experts;
    }
}

}  // namespace dsv4b

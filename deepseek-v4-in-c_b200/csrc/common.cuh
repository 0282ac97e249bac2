// common.cuh - shared device helpers for the B200 decode backend (sm_100a).
//
// Weight formats are the reference's (src/core/dsv4_quant.h:74-164): e4m3fn
// codes with E8M0 128x128 block scales, e2m1 codes two per byte (even element
// in the LOW nibble) with E8M0 1x32 scales, bf16, f32. The helpers here decode
// with the hardware converters (cvt.rn.f16x2.e4m3x2 / .e2m1x2), which are
// exact: every e4m3 and e2m1 value, subnormals included, is representable in
// f16, and every f16 in f32 (the tensor-core FP4 path places e2m1 codes into
// f16 bit fields itself, gemv_mma.cuh).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_fp4.h>
#include <stdint.h>
#include <stdio.h>

#define DSV4B_WF32 0
#define DSV4B_WBF16 1
#define DSV4B_WFP8 2
#define DSV4B_WFP4 3

namespace dsv4b {

// ------------------------------------------------------------- decoding ---

// E8M0 byte -> float: 2^(b-127); 0 is the subnormal 2^-127, 0xFF is NaN
// (dsv4_quant.h:74-88).
__device__ __forceinline__ float e8m0(uint8_t b)
{
    uint32_t u = (uint32_t)b << 23;
    u = (b == 0u) ? 0x00400000u : u;
    u = (b == 0xFFu) ? 0x7FC00000u : u;
    return __uint_as_float(u);
}

// Two e4m3 codes (low byte = first element) -> two floats.
__device__ __forceinline__ float2 e4m3x2(uint16_t v)
{
    __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)v, __NV_E4M3);
    return __half22float2(*reinterpret_cast<__half2 *>(&h));
}

// One byte of two e2m1 codes (low nibble = first element) -> two floats.
__device__ __forceinline__ float2 e2m1x2(uint8_t v)
{
    __half2_raw h = __nv_cvt_fp4x2_to_halfraw2((__nv_fp4x2_storage_t)v, __NV_E2M1);
    return __half22float2(*reinterpret_cast<__half2 *>(&h));
}

__device__ __forceinline__ float2 bf16x2(uint32_t v)
{
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
}

// ------------------------------------------------------------------ loads ---

// Streaming 16-byte weight load: read-only path, no L1 allocation. Weights are
// touched once per launch, so caching them in L1 would only evict x.
__device__ __forceinline__ uint4 ld_stream16(const void *p)
{
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

// Activations written by the previous kernel: coherent L2 loads. Under
// programmatic dependent launch a kernel is already running while its
// predecessor writes, so the read-only (.nc) path, whose contract is data
// unchanged for the kernel's lifetime, is reserved for weights.
__device__ __forceinline__ float4 ld_f4(const float *p)
{
    return __ldcg(reinterpret_cast<const float4 *>(p));
}
__device__ __forceinline__ float2 ld_f2(const float *p)
{
    return __ldcg(reinterpret_cast<const float2 *>(p));
}
__device__ __forceinline__ float ld_act(const float *p) { return __ldcg(p); }
__device__ __forceinline__ double ld_act_d(const double *p) { return __ldcg(p); }

// Packed two-lane FMA (Blackwell FFMA2): c.x += a.x*b.x, c.y += a.y*b.y, each
// lane a single correctly rounded fma.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c)
{
    uint64_t d;
    const uint64_t ua = (uint64_t)__float_as_uint(a.x) | ((uint64_t)__float_as_uint(a.y) << 32);
    const uint64_t ub = (uint64_t)__float_as_uint(b.x) | ((uint64_t)__float_as_uint(b.y) << 32);
    const uint64_t uc = (uint64_t)__float_as_uint(c.x) | ((uint64_t)__float_as_uint(c.y) << 32);
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(ua), "l"(ub), "l"(uc));
    return make_float2(__uint_as_float((uint32_t)d), __uint_as_float((uint32_t)(d >> 32)));
}

__device__ __forceinline__ double warp_sum_d(double v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum_f(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_max_f(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ---------------------------------------------- programmatic dependent launch
// Kernels of a decode step are launched with programmatic stream
// serialization: each lets its dependents be scheduled as soon as all of its
// blocks are running (pdl_trigger), and waits for its predecessor to finish
// and flush (pdl_wait) before reading anything the predecessor wrote or
// writing anything it may still read. Launched without the attribute, both
// are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Interleaved-pair RoPE of the last rd dims of a width-wide vector at table
// row `pos` (src/core/dsv4_rope.c:106-120); inverse negates the sine.
__device__ __forceinline__ void rope_tail(float *v, int width, int rd, const float *cs, const float *sn,
                                          int pos, int inverse)
{
    float *tail = v + (width - rd);
    const int half = rd / 2;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const float re = tail[2 * i], im = tail[2 * i + 1];
        const float ci = cs[(size_t)pos * half + i];
        const float si = inverse ? -sn[(size_t)pos * half + i] : sn[(size_t)pos * half + i];
        tail[2 * i] = __fsub_rn(__fmul_rn(re, ci), __fmul_rn(im, si));
        tail[2 * i + 1] = __fadd_rn(__fmul_rn(re, si), __fmul_rn(im, ci));
    }
}

}  // namespace dsv4b

#define DSV4B_CUDA_OK(call)                                                     \
    do {                                                                       \
        cudaError_t e_ = (call);                                               \
        if (e_ != cudaSuccess) {                                               \
            fprintf(stderr, "dsv4_b200: %s failed: %s (%s:%d)\n", #call,       \
                    cudaGetErrorString(e_), __FILE__, __LINE__);               \
            return -1;                                                         \
        }                                                                      \
    } while (0)

// jdg_common.cuh — device helpers shared by the decode kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define JDG_FULL 0xffffffffu

// device error flags (bitwise OR into the engine's error word)
enum {
    JDG_ERR_TOKEN = 1,   // token id outside [0, vocab)
    JDG_ERR_POS = 2,     // position outside [0, max_seq)
    JDG_ERR_ROUTE = 4,   // election produced an invalid expert slot
    JDG_ERR_SHAPE = 8,   // a kernel met a shape it does not support
    JDG_ERR_TIMEOUT = 16,  // a bounded wait on an asynchronous copy ran out
};

// Split-K partial tiles of a single-segment tensor-core product that the consumer sums
// itself (no separate reduce launch): tile (row tile tt, column tile rt) holds
// [ks][128 tokens][128 columns] at tile = tt * rtiles + rt.  part null: none.
constexpr int kSplitTile = 128;
constexpr int kSplitMax = 8;  // split ways at most
struct SplitPart {
    const float *part;
    int ks, rtiles;
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(JDG_FULL, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(JDG_FULL, v, o));
    return v;
}
// streaming 128-bit load: weights are read once per step, keep them out of L1
__device__ __forceinline__ float4 ld_stream4(const float *p) {
    float4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint4 ld_stream_u4(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ float dot4(float4 a, float4 b, float acc) {
    acc = fmaf(a.x, b.x, acc);
    acc = fmaf(a.y, b.y, acc);
    acc = fmaf(a.z, b.z, acc);
    acc = fmaf(a.w, b.w, acc);
    return acc;
}
// janusdoe.c:498 silu_f
__device__ __forceinline__ float silu_ref(float x) { return x / (1.0f + expf(-x)); }

// janusdoe.c:191-192 xorshift64 and its 31-bit uniform
__device__ __forceinline__ uint64_t xs_next(uint64_t &s) {
    uint64_t x = s;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    s = x;
    return x;
}
__device__ __forceinline__ float xs_uniform(uint64_t &s) {
    return (float)(xs_next(s) & 0x7FFFFFFFull) / (float)0x7FFFFFFF;
}

// exact IEEE half -> float (janusdoe.c:2545): __half2float is exact for every half
__device__ __forceinline__ float h2f(uint16_t h) {
    float f;
    asm("{ .reg .b16 t; mov.b16 t, %1; cvt.f32.f16 %0, t; }" : "=f"(f) : "h"(h));
    return f;
}

// block-wide sum for blockDim.x a multiple of 32 (<= 1024); red has >= 32 floats
__device__ __forceinline__ float block_sum(float v, float *red) {
    int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float t = 0.f;
    if (wid == 0) {
        t = lane < nw ? red[lane] : 0.f;
        t = warp_sum(t);
        if (lane == 0) red[0] = t;
    }
    __syncthreads();
    return red[0];
}

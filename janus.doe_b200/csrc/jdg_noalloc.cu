// jdg_noalloc.cu — vocabulary projection + greedy pick that allocates no device memory.
//
// Some callers cannot call cudaMalloc: a host program whose device memory all comes from
// another allocator (a framework's caching allocator, a preallocated pool shared with other
// code, a sandbox that only hands out buffers it owns).  jdg_logits_argmax_noalloc lets such
// a caller run the LM head and the greedy pick on buffers it already has.  It is the
// batch-1 LM-head kernel of the decode step in a form that takes device pointers: each CTA
// projects 16 rows, keeps its (max, first index), and the last CTA to finish reduces those
// partials.  The partials and the completion ticket live in one file-scope __device__ array
// instead of a cudaMalloc'd buffer.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/jdgpu.h"
#include "jdg_common.cuh"
#include "jdg_engine.h"

namespace {

constexpr int kNaRowsPerCta = 16;   // 8 warps x 2 rows
constexpr int kNaMaxCtas = 8192;    // scratch capacity: 8192 CTAs -> 131072 rows
constexpr int kNaMaxCols = 16384;   // x staged in shared memory (64 KB)

struct NoAllocScratch {
    float val[kNaMaxCtas];
    int idx[kNaMaxCtas];
    unsigned ticket;
};

// Shared by every call on a device and kept until the process exits (about 64 KB per GPU
// that loads the library).  Host code must not take its address directly: on the host the
// name is only a stand-in, so the device address is looked up with cudaGetSymbolAddress.
static __device__ __align__(256) NoAllocScratch g_na_scratch;

constexpr int kNaMaxDevices = 64;
std::mutex g_na_mu;
NoAllocScratch *g_na_ptr[kNaMaxDevices] = {};

__global__ __launch_bounds__(256) void k_logits_argmax(const float *__restrict__ W, const float *__restrict__ x, int rows,
                                                       int cols, float *__restrict__ logits, int *__restrict__ argmax,
                                                       NoAllocScratch *scr) {
    extern __shared__ __align__(16) float xs[];
    __shared__ float bv_s[8];
    __shared__ int bi_s[8];
    __shared__ unsigned s_ticket;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < cols / 4; i += blockDim.x)
        reinterpret_cast<float4 *>(xs)[i] = reinterpret_cast<const float4 *>(x)[i];
    __syncthreads();
    float val = -INFINITY;
    int vi = 0x7fffffff;
    const int row0 = blockIdx.x * kNaRowsPerCta + warp * 2;
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const int row = row0 + r;
        if (row >= rows) break;
        const float *wr = W + (size_t)row * cols;
        float acc = 0.f;
        for (int k4 = lane; k4 < cols / 4; k4 += 32)
            acc = dot4(ld_stream4(wr + 4 * k4), reinterpret_cast<const float4 *>(xs)[k4], acc);
        acc = warp_sum(acc);
        if (lane == 0) logits[row] = acc;
        if (acc > val) {  // rows ascend within a warp: the first maximum is kept
            val = acc;
            vi = row;
        }
    }
    if (lane == 0) {
        bv_s[warp] = val;
        bi_s[warp] = vi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float bv = bv_s[0];
        int bi = bi_s[0];
        for (int q = 1; q < 8; q++)
            if (bv_s[q] > bv || (bv_s[q] == bv && bi_s[q] < bi)) {
                bv = bv_s[q];
                bi = bi_s[q];
            }
        scr->val[blockIdx.x] = bv;
        scr->idx[blockIdx.x] = bi;
        __threadfence();
        s_ticket = atomicAdd(&scr->ticket, 1u);
    }
    __syncthreads();
    if (s_ticket != gridDim.x - 1) return;
    // last CTA: first-index maximum over the per-CTA partials
    __threadfence();
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int q = threadIdx.x; q < (int)gridDim.x; q += blockDim.x) {
        const float v = __ldcg(&scr->val[q]);
        const int ix = __ldcg(&scr->idx[q]);
        if (v > bv || (v == bv && ix < bi)) {
            bv = v;
            bi = ix;
        }
    }
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(JDG_FULL, bv, o);
        const int oi = __shfl_xor_sync(JDG_FULL, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if (lane == 0) {
        bv_s[warp] = bv;
        bi_s[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int q = 1; q < 8; q++)
            if (bv_s[q] > bv_s[0] || (bv_s[q] == bv_s[0] && bi_s[q] < bi_s[0])) {
                bv_s[0] = bv_s[q];
                bi_s[0] = bi_s[q];
            }
        *argmax = bi_s[0] == 0x7fffffff ? 0 : bi_s[0];
        scr->ticket = 0;
    }
}

// Device address of the scratch array for the current device, looked up once per device
// (with that device current) and cached.
int na_scratch(NoAllocScratch **out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kNaMaxDevices) {
        jdg_set_err(nullptr, "jdg_logits_argmax_noalloc: no usable current device (%s)",
                 cudaGetErrorString(e));
        return JD_ECUDA;
    }
    std::lock_guard<std::mutex> lk(g_na_mu);
    if (!g_na_ptr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_na_scratch);
        if (e != cudaSuccess || !p) {
            jdg_set_err(nullptr, "jdg_logits_argmax_noalloc: cudaGetSymbolAddress failed: %s",
                     cudaGetErrorString(e));
            return JD_ECUDA;
        }
        e = cudaFuncSetAttribute(k_logits_argmax, cudaFuncAttributeMaxDynamicSharedMemorySize, kNaMaxCols * 4);
        if (e != cudaSuccess) {
            jdg_set_err(nullptr, "jdg_logits_argmax_noalloc: cudaFuncSetAttribute failed: %s",
                     cudaGetErrorString(e));
            return JD_ECUDA;
        }
        g_na_ptr[dev] = (NoAllocScratch *)p;
    }
    *out = g_na_ptr[dev];
    return JD_OK;
}

}  // namespace

extern "C" int jdg_logits_argmax_noalloc_check(const void *W_dev, const void *x_dev, int rows, int cols,
                                               const void *logits_dev, const void *argmax_dev) {
    // Pure host arithmetic on the arguments: no CUDA call, no dereference.
    if (!W_dev || !x_dev || !logits_dev || !argmax_dev || rows < 1 || cols < 4 || cols % 4) {
        jdg_set_err(nullptr, "jdg_logits_argmax_noalloc: bad arguments (rows %d, cols %d)", rows, cols);
        return JD_EINVAL;
    }
    // W rows and x are read as 16-byte vectors: a misaligned view would fault on the GPU
    if (((uintptr_t)W_dev | (uintptr_t)x_dev) & 15u) {
        jdg_set_err(nullptr, "jdg_logits_argmax_noalloc: W_dev and x_dev must be 16-byte aligned (%p, %p)", W_dev,
                    x_dev);
        return JD_EINVAL;
    }
    const long ctas = ((long)rows + kNaRowsPerCta - 1) / kNaRowsPerCta;
    if (ctas > kNaMaxCtas || cols > kNaMaxCols) {
        jdg_set_err(nullptr,
                    "jdg_logits_argmax_noalloc: %d x %d exceeds the fixed scratch (at most %d rows and %d columns)",
                    rows, cols, kNaMaxCtas * kNaRowsPerCta, kNaMaxCols);
        return JD_EINVAL;
    }
    return JD_OK;
}

extern "C" int jdg_logits_argmax_noalloc(const float *W_dev, const float *x_dev, int rows, int cols, float *logits_dev,
                                         int *argmax_dev, void *stream) {
    int rc = jdg_logits_argmax_noalloc_check(W_dev, x_dev, rows, cols, logits_dev, argmax_dev);
    if (rc != JD_OK) return rc;
    const int ctas = (rows + kNaRowsPerCta - 1) / kNaRowsPerCta;
    NoAllocScratch *scr = nullptr;
    rc = na_scratch(&scr);
    if (rc != JD_OK) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    if (st) {  // the scratch address belongs to the current device: so must the stream
        int cur = -1, sdev = -1;
        cudaError_t ge = cudaGetDevice(&cur);
        if (ge == cudaSuccess) ge = cudaStreamGetDevice(st, &sdev);
        if (ge != cudaSuccess || sdev != cur) {
            jdg_set_err(nullptr, "jdg_logits_argmax_noalloc: the stream is not on the current device (%d vs %d%s%s)",
                        sdev, cur, ge != cudaSuccess ? ": " : "", ge != cudaSuccess ? cudaGetErrorString(ge) : "");
            return JD_EINVAL;
        }
    }
    // the ticket must start at zero; a memset allocates nothing
    cudaError_t e = cudaMemsetAsync(&scr->ticket, 0, sizeof(unsigned), st);
    if (e == cudaSuccess) {
        k_logits_argmax<<<ctas, 256, (size_t)cols * 4, st>>>(W_dev, x_dev, rows, cols, logits_dev, argmax_dev, scr);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) {
        jdg_set_err(nullptr, "jdg_logits_argmax_noalloc: launch failed: %s", cudaGetErrorString(e));
        return JD_ECUDA;
    }
    return JD_OK;
}

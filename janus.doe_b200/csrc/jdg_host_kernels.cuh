// jdg_host_kernels.cuh — kernels of the host GGUF path: dequant-fused GEMV (one token) and
// GEMM (a batch of tokens) over repacked Q8_0 / Q4_K / f32 weights, the LoRA parliament
// deltas, and small helpers.
//
// Device layout of packed weights (repacked at upload, lossless):
//   Q8_0: q[row][K] int8 codes; s[row][K/32] f16 scales d         (34 bytes / 32 weights)
//   Q4_K: q[row][K/2] bytes (each 144-byte superblock's 128 code bytes, in file order);
//         s[row][K/256] 16-byte headers {f16 d, f16 dmin, 12 packed 6-bit scales/mins}
//   Q6_K: q = [row][K/2] low-nibble bytes then [row][K/4] 2-bit high parts (file order per
//         superblock); s[row][K/256] 32-byte headers {16 int8 scales, f16 d}  (7 bits/weight)
//   F32:  q[row][K] floats
// Q4_0 / Q5_0 arrive in the Q8_0 layout (their codes minus 8 / 16 are int8 codes with the
// same per-32 f16 scale) and F16 as F32: both exact.
// The value of a weight is exactly the reference's dequantisation (janusdoe.c:2566-2585):
//   Q8_0: d * q;   Q4_K: (d*s_j) * q - (dmin*m_j) for sub-block j.
#pragma once
#include "jd_quant.h"
#include "jdg_kernels.cuh"

namespace jdg {

struct QW {
    int dt;            // JD_F32 (0), JD_Q8_0 (8), JD_Q4_K (12), JD_Q6_K (14)
    int rows, cols;
    const uint8_t *q;
    const uint8_t *s;
};

// 6-bit scale and minimum of Q4_K sub-block j from the 12 packed header bytes (jd_quant.h)
__device__ __forceinline__ void smk4(int j, const uint8_t *sc, int &s, int &m) { jdq_q4k_scale_min(sc, j, &s, &m); }
// exact small non-negative integer -> float (no I2F): 2^23 + n, then subtract 2^23
__device__ __forceinline__ float u2f_small(uint32_t n) { return __uint_as_float(0x4B000000u | n) - 8388608.0f; }
__device__ __forceinline__ float s8f(uint32_t word, int byte) {
    // signed byte -> float: bias to unsigned, exact integer conversion, remove the bias
    uint32_t b = ((word >> (8 * byte)) & 0xFFu) ^ 0x80u;
    return u2f_small(b) - 128.0f;
}

// ------------------------------------------------------------------------------------
// GEMV, one token: y[row] (epi) W[row] . x.  One warp per row (two rows for SWIGLU),
// x staged in shared memory with sums of 16 (Q4_K min terms).  K: multiple of 32 (Q8_0)
// or 256 (Q4_K).
// Epilogue: EPI_STORE, EPI_ADD (y += acc * alpha), EPI_SWIGLU (rows 2i, 2i+1).
struct QGemvArgs {
    QW w;
    const float *x;
    float *y;
    float alpha;
};

template <int DT>
__device__ __forceinline__ float qrow_dot(const QW &w, int row, const float *xs, const float *xsum, int lane) {
    const int K = w.cols;
    float acc = 0.f;
    if (DT == 8) {
        const uint8_t *qr = w.q + (size_t)row * K;
        const uint16_t *sr = reinterpret_cast<const uint16_t *>(w.s) + (size_t)row * (K / 32);
#pragma unroll 4
        for (int e0 = lane * 16; e0 < K; e0 += 512) {
            uint4 qv = ld_stream_u4(qr + e0);
            const float d = h2f(sr[e0 >> 5]);
            const float4 *x4 = reinterpret_cast<const float4 *>(xs + e0);
            float s = 0.f;
            uint32_t wd[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
            for (int c = 0; c < 4; c++) {
                float4 xv = x4[c];
                s = fmaf(s8f(wd[c], 0), xv.x, s);
                s = fmaf(s8f(wd[c], 1), xv.y, s);
                s = fmaf(s8f(wd[c], 2), xv.z, s);
                s = fmaf(s8f(wd[c], 3), xv.w, s);
            }
            acc = fmaf(d, s, acc);
        }
    } else if (DT == 12) {
        const uint8_t *qr = w.q + (size_t)row * (K / 2);
        const uint8_t *hr = w.s + (size_t)row * (K / 256) * 16;
#pragma unroll 4
        for (int byte0 = lane * 16; byte0 < K / 2; byte0 += 512) {
            // a pass covers 512 code bytes (1024 weights); this lane's 16 bytes lie in
            // superblock sb, chunk c (64 weights), at l0 in {0, 16}
            const int sb = byte0 >> 7, o = byte0 & 127, c = o >> 5, l0 = o & 31;
            uint4 qv = ld_stream_u4(qr + byte0);
            const uint4 hv = *reinterpret_cast<const uint4 *>(hr + (size_t)sb * 16);
            const uint8_t *hb = reinterpret_cast<const uint8_t *>(&hv);
            const float d = h2f((uint16_t)(hb[0] | (hb[1] << 8))), dmin = h2f((uint16_t)(hb[2] | (hb[3] << 8)));
            int s0, m0, s1, m1;
            smk4(2 * c, hb + 4, s0, m0);
            smk4(2 * c + 1, hb + 4, s1, m1);
            const float d1 = d * (float)s0, mm1 = dmin * (float)m0, d2 = d * (float)s1, mm2 = dmin * (float)m1;
            const int xb = sb * 256 + 64 * c + l0;
            const float4 *xl = reinterpret_cast<const float4 *>(xs + xb);
            const float4 *xh = reinterpret_cast<const float4 *>(xs + xb + 32);
            uint32_t wd[4] = {qv.x, qv.y, qv.z, qv.w};
            float sl = 0.f, sh = 0.f;
#pragma unroll
            for (int cc = 0; cc < 4; cc++) {
                float4 a = xl[cc], b = xh[cc];
                uint32_t v = wd[cc];
                sl = fmaf(u2f_small(v & 15u), a.x, sl);
                sh = fmaf(u2f_small((v >> 4) & 15u), b.x, sh);
                sl = fmaf(u2f_small((v >> 8) & 15u), a.y, sl);
                sh = fmaf(u2f_small((v >> 12) & 15u), b.y, sh);
                sl = fmaf(u2f_small((v >> 16) & 15u), a.z, sl);
                sh = fmaf(u2f_small((v >> 20) & 15u), b.z, sh);
                sl = fmaf(u2f_small((v >> 24) & 15u), a.w, sl);
                sh = fmaf(u2f_small(v >> 28), b.w, sh);
            }
            // sum over this lane's 16 elements of x for the min terms
            const float xs_l = xsum[(xb >> 4)], xs_h = xsum[(xb + 32) >> 4];
            acc = fmaf(d1, sl, acc);
            acc = fmaf(-mm1, xs_l, acc);
            acc = fmaf(d2, sh, acc);
            acc = fmaf(-mm2, xs_h, acc);
        }
    } else if (DT == 14) {
        // Q6_K: a lane takes 16 low-nibble bytes of one half superblock (bytes b..b+15 of its
        // 64) and the 16 high-part bytes they share: 16 weights of quarter u = b/32 (low
        // nibbles) and 16 of quarter u + 2 (high nibbles), one int8 scale each
        const uint8_t *qr = w.q + (size_t)row * (K / 2);
        const uint8_t *hr = w.q + (size_t)w.rows * (K / 2) + (size_t)row * (K / 4);
        const uint8_t *sr = w.s + (size_t)row * (K / 256) * 32;
#pragma unroll 2
        for (int byte0 = lane * 16; byte0 < K / 2; byte0 += 512) {
            const int sb = byte0 >> 7, o = byte0 & 127, hf = o >> 6, b = o & 63, u = b >> 5, l0 = b & 31;
            const uint4 lv = ld_stream_u4(qr + byte0);
            const uint4 hv = ld_stream_u4(hr + (size_t)sb * 64 + 32 * hf + l0);
            const uint8_t *hd = sr + (size_t)sb * 32;
            const float d = h2f((uint16_t)(hd[16] | (hd[17] << 8)));
            const float dl = d * (float)(int8_t)hd[8 * hf + (l0 >> 4) + 2 * u];
            const float dh = d * (float)(int8_t)hd[8 * hf + (l0 >> 4) + 2 * (u + 2)];
            const int e0 = sb * 256 + 128 * hf + b;
            const float4 *xl = reinterpret_cast<const float4 *>(xs + e0);
            const float4 *xh = reinterpret_cast<const float4 *>(xs + e0 + 64);
            const uint32_t lw[4] = {lv.x, lv.y, lv.z, lv.w}, hw[4] = {hv.x, hv.y, hv.z, hv.w};
            float sl = 0.f, sh = 0.f;
#pragma unroll
            for (int cc = 0; cc < 4; cc++) {
                const float4 a4 = xl[cc], b4 = xh[cc];
                const float av[4] = {a4.x, a4.y, a4.z, a4.w}, bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const uint32_t qlb = (lw[cc] >> (8 * j)) & 0xFFu, qhb = (hw[cc] >> (8 * j)) & 0xFFu;
                    const uint32_t q0 = (qlb & 15u) | (((qhb >> (2 * u)) & 3u) << 4);
                    const uint32_t q1 = (qlb >> 4) | (((qhb >> (2 * u + 4)) & 3u) << 4);
                    sl = fmaf(u2f_small(q0) - 32.0f, av[j], sl);
                    sh = fmaf(u2f_small(q1) - 32.0f, bv[j], sh);
                }
            }
            acc = fmaf(dl, sl, acc);
            acc = fmaf(dh, sh, acc);
        }
    } else {
        const float *wr = reinterpret_cast<const float *>(w.q) + (size_t)row * K;
#pragma unroll 4
        for (int k4 = lane; k4 < K / 4; k4 += 32)
            acc = dot4(ld_stream4(wr + 4 * k4), reinterpret_cast<const float4 *>(xs)[k4], acc);
    }
    return warp_sum(acc);
}

template <int DT, int EPI>
static __global__ __launch_bounds__(256) void k_qgemv(QGemvArgs a) {
    extern __shared__ __align__(16) float xs[];  // [K] then [K/16] sums of 16
    const int K = a.w.cols;
    float *xsum = xs + K;
    for (int i = threadIdx.x; i < K / 4; i += blockDim.x)
        reinterpret_cast<float4 *>(xs)[i] = reinterpret_cast<const float4 *>(a.x)[i];
    __syncthreads();
    if (DT == 12)
        for (int g = threadIdx.x; g < K / 16; g += blockDim.x) {
            float t = 0.f;
#pragma unroll
            for (int i = 0; i < 16; i++) t += xs[16 * g + i];
            xsum[g] = t;
        }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (EPI == EPI_SWIGLU) {
        const int i = blockIdx.x * nw + warp;  // hidden unit: rows 2i (gate), 2i+1 (up)
        if (2 * i + 1 >= a.w.rows) return;
        float g = qrow_dot<DT>(a.w, 2 * i, xs, xsum, lane);
        float u = qrow_dot<DT>(a.w, 2 * i + 1, xs, xsum, lane);
        // janusdoe.c:3272: gate[i] / (1 + expf(-gate[i])) * up[i]
        if (lane == 0) a.y[i] = __fmul_rn(silu_ref(g), u);
    } else {
        const int row = blockIdx.x * nw + warp;
        if (row >= a.w.rows) return;
        float v = qrow_dot<DT>(a.w, row, xs, xsum, lane);
        if (lane == 0) {
            if (EPI == EPI_ADD) a.y[row] = __fadd_rn(a.y[row], __fmul_rn(v, a.alpha));
            else a.y[row] = v;
        }
    }
}

// ------------------------------------------------------------------------------------
// GEMM over a batch: C[m][n] (epi) sum_k X[m][k] W[n][k].  Tile 32 tokens x 64 rows,
// K step 256: the W tile is dequantised into shared memory as f32 (exact values), the X
// tile staged alongside; 256 threads, thread tile 2 tokens x 4 rows.
struct QGemmArgs {
    QW w;
    const float *X;
    int ldx, M;
    float *C;
    int ldc;
    float alpha;
};
template <int DT>
__device__ __forceinline__ void dequant_tile(const QW &w, int n0, int k0, float (*Ws)[257], int tid) {
    // 64 rows x 256 weights
    if (DT == 8) {
        // 64 rows x 8 blocks of 32: thread t handles (row t/4, blocks 2*(t%4), 2*(t%4)+1)
        const int r = tid >> 2, bq = (tid & 3) * 2;
        const int row = n0 + r;
        for (int bb = 0; bb < 2; bb++) {
            const int b = bq + bb;
            if (row < w.rows) {
                const uint8_t *qp = w.q + (size_t)row * w.cols + k0 + 32 * b;
                const float d = h2f(reinterpret_cast<const uint16_t *>(w.s)[(size_t)row * (w.cols / 32) + (k0 >> 5) + b]);
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    uint4 v = *reinterpret_cast<const uint4 *>(qp + 16 * c);
                    uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int j = 0; j < 16; j++) Ws[r][32 * b + 16 * c + j] = d * s8f(wd[j >> 2], j & 3);
                }
            } else {
                for (int j = 0; j < 32; j++) Ws[r][32 * b + j] = 0.f;
            }
        }
    } else if (DT == 12) {
        // 64 rows x 1 superblock: thread t handles row t/4, chunk t%4 (64 weights)
        const int r = tid >> 2, c = tid & 3, row = n0 + r;
        if (row < w.rows) {
            const uint8_t *qp = w.q + (size_t)row * (w.cols / 2) + (k0 / 2) + 32 * c;
            const uint8_t *hb = w.s + ((size_t)row * (w.cols / 256) + (k0 >> 8)) * 16;
            const float d = h2f((uint16_t)(hb[0] | (hb[1] << 8))), dmin = h2f((uint16_t)(hb[2] | (hb[3] << 8)));
            int s0, m0, s1, m1;
            smk4(2 * c, hb + 4, s0, m0);
            smk4(2 * c + 1, hb + 4, s1, m1);
            const float d1 = d * (float)s0, mm1 = dmin * (float)m0, d2 = d * (float)s1, mm2 = dmin * (float)m1;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                uint4 v = *reinterpret_cast<const uint4 *>(qp + 16 * h);
                uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    uint32_t byte = (wd[j >> 2] >> (8 * (j & 3))) & 0xFFu;
                    Ws[r][64 * c + 16 * h + j] = __fsub_rn(__fmul_rn(d1, u2f_small(byte & 15u)), mm1);
                    Ws[r][64 * c + 32 + 16 * h + j] = __fsub_rn(__fmul_rn(d2, u2f_small(byte >> 4)), mm2);
                }
            }
        } else {
            for (int j = 0; j < 64; j++) Ws[r][64 * c + j] = 0.f;
        }
    } else if (DT == 14) {
        // 64 rows x 1 superblock: thread t handles row t/4; c = t%4 picks half c/2 and its low
        // (quarters 0, 1) or high (quarters 2, 3) nibbles: 64 weights, value (d*sc)*(q - 32)
        const int r = tid >> 2, c = tid & 3, row = n0 + r, hf = c >> 1, part = c & 1;
        if (row < w.rows) {
            const int K = w.cols, sb = k0 >> 8;
            const uint8_t *ql = w.q + (size_t)row * (K / 2) + (size_t)sb * 128 + 64 * hf;
            const uint8_t *qh = w.q + (size_t)w.rows * (K / 2) + (size_t)row * (K / 4) + (size_t)sb * 64 + 32 * hf;
            const uint8_t *hd = w.s + ((size_t)row * (K / 256) + sb) * 32;
            const float d = h2f((uint16_t)(hd[16] | (hd[17] << 8)));
#pragma unroll 4
            for (int b = 0; b < 64; b++) {
                const int u = (b >> 5) + 2 * part;
                const uint32_t qlb = ql[b], qhb = qh[b & 31];
                const uint32_t q = (part ? qlb >> 4 : qlb & 15u) | (((qhb >> (2 * u)) & 3u) << 4);
                const float ds = __fmul_rn(d, (float)(int8_t)hd[8 * hf + ((b & 31) >> 4) + 2 * u]);
                Ws[r][128 * hf + 64 * part + b] = __fmul_rn(ds, u2f_small(q) - 32.0f);
            }
        } else {
            for (int j = 0; j < 64; j++) Ws[r][64 * c + j] = 0.f;
        }
    } else {
        const int r = tid >> 2, c = tid & 3, row = n0 + r;
        const float *wp = reinterpret_cast<const float *>(w.q) + (size_t)row * w.cols + k0 + 64 * c;
        for (int j = 0; j < 64; j += 4) {
            float4 v = row < w.rows ? *reinterpret_cast<const float4 *>(wp + j) : make_float4(0.f, 0.f, 0.f, 0.f);
            Ws[r][64 * c + j] = v.x;
            Ws[r][64 * c + j + 1] = v.y;
            Ws[r][64 * c + j + 2] = v.z;
            Ws[r][64 * c + j + 3] = v.w;
        }
    }
}

template <int DT, int EPI>
static __global__ __launch_bounds__(256) void k_qgemm(QGemmArgs a) {
    extern __shared__ __align__(16) float smem[];
    float(*Ws)[257] = reinterpret_cast<float(*)[257]>(smem);           // [64][257]
    float(*Xs)[257] = reinterpret_cast<float(*)[257]>(smem + 64 * 257);  // [32][257]
    const int n0 = blockIdx.x * 64, m0 = blockIdx.y * 32, tid = threadIdx.x;
    const int tm = tid >> 4, tn = tid & 15;  // tokens 2*tm.., rows tn + 16*j
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    for (int k0 = 0; k0 < a.w.cols; k0 += 256) {
        __syncthreads();
        dequant_tile<DT>(a.w, n0, k0, Ws, tid);
        for (int i = tid; i < 32 * 64; i += 256) {
            int m = i >> 6, k4 = i & 63;
            float4 v = (m0 + m < a.M) ? *reinterpret_cast<const float4 *>(a.X + (size_t)(m0 + m) * a.ldx + k0 + 4 * k4)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
            Xs[m][4 * k4] = v.x;
            Xs[m][4 * k4 + 1] = v.y;
            Xs[m][4 * k4 + 2] = v.z;
            Xs[m][4 * k4 + 3] = v.w;
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < 256; k++) {
            float x0 = Xs[2 * tm][k], x1 = Xs[2 * tm + 1][k];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                float wv = Ws[tn + 16 * j][k];
                acc[0][j] = fmaf(x0, wv, acc[0][j]);
                acc[1][j] = fmaf(x1, wv, acc[1][j]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const int m = m0 + 2 * tm + i;
        float *c = a.C + (size_t)m * a.ldc;
        if (EPI == EPI_SWIGLU) {
            // rows (2i, 2i+1) live in threads tn and tn^1 of the same half-warp; every lane
            // takes part in the shuffle, only valid tokens store
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int n = n0 + tn + 16 * j;
                float other = __shfl_xor_sync(JDG_FULL, acc[i][j], 1);
                if (m < a.M && (tn & 1) == 0 && n + 1 < a.w.rows) c[n >> 1] = __fmul_rn(silu_ref(acc[i][j]), other);
            }
        } else {
            if (m >= a.M) continue;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int n = n0 + tn + 16 * j;
                if (n < a.w.rows) {
                    if (EPI == EPI_ADD) c[n] = __fadd_rn(c[n], __fmul_rn(acc[i][j], a.alpha));
                    else c[n] = acc[i][j];
                }
            }
        }
    }
}

// ------------------------------------------------------------------------------------
// LoRA parliament (janusdoe.c:3281-3303).  t[b][ki][r] = B_e[r] . xn[b] for the elected
// experts; grid (R, 16, B), one dot of length D per CTA.
static __global__ __launch_bounds__(256) void k_lora_t(const float *__restrict__ loraB, int R, int D, const int *__restrict__ kcnt,
                                                const int *__restrict__ sel, const float *__restrict__ xn,
                                                float *__restrict__ t) {
    __shared__ float red[32];
    const int r = blockIdx.x, ki = blockIdx.y, b = blockIdx.z;
    if (ki >= kcnt[b]) return;
    const int e = sel[b * kMaxE + ki];
    const float *Br = loraB + ((size_t)e * R + r) * D;
    const float *xr = xn + (size_t)b * D;
    float s = 0.f;
    for (int j = threadIdx.x * 4; j < D; j += blockDim.x * 4) {
        float4 bv = *reinterpret_cast<const float4 *>(Br + j), xv = *reinterpret_cast<const float4 *>(xr + j);
        s = dot4(bv, xv, s);
    }
    s = block_sum(s, red);
    if (threadIdx.x == 0) t[((size_t)b * kMaxE + ki) * R + r] = s;
}
// x[b][i] += (alpha * w_ki) * (A_e[i] . t_ki), experts in election order; grid (D/256, B)
static __global__ __launch_bounds__(256) void k_lora_apply(const float *__restrict__ loraA, int R, int D, float alpha,
                                                    const int *__restrict__ kcnt, const int *__restrict__ sel,
                                                    const float *__restrict__ selw, const float *__restrict__ t,
                                                    float *__restrict__ x) {
    const int b = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= D) return;
    const int k = kcnt[b];
    float xi = x[(size_t)b * D + i];
    for (int ki = 0; ki < k; ki++) {
        const int e = sel[b * kMaxE + ki];
        const float *Ar = loraA + ((size_t)e * D + i) * R;
        const float *tr = t + ((size_t)b * kMaxE + ki) * R;
        float s = 0.f;
        for (int r = 0; r < R; r++) s = fmaf(Ar[r], tr[r], s);
        const float w = __fmul_rn(alpha, selw[b * kMaxE + ki]);
        xi = __fadd_rn(xi, __fmul_rn(w, s));
    }
    x[(size_t)b * D + i] = xi;
}

// x += y (all-reduced partial sums in tensor-parallel runs)
static __global__ void k_add(float *__restrict__ x, const float *__restrict__ y, size_t n) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = __fadd_rn(x[i], y[i]);
}

// vocab-parallel greedy pick: each rank's (max, first index) per sequence
static __global__ __launch_bounds__(1024) void k_argmax_part(const float *__restrict__ logits, int V, int ldl, int off,
                                                      float *__restrict__ out_v, int *__restrict__ out_i) {
    const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __shared__ float rv[32];
    __shared__ int ri[32];
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < V; i += blockDim.x) {
        float v = logits[(size_t)b * ldl + i];
        if (v > bv) {
            bv = v;
            bi = i;
        }
    }
    for (int o = 16; o; o >>= 1) {
        float ov = __shfl_xor_sync(JDG_FULL, bv, o);
        int oi = __shfl_xor_sync(JDG_FULL, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if (lane == 0) {
        rv[warp] = bv;
        ri[warp] = bi;
    }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++)
            if (rv[w] > bv || (rv[w] == bv && ri[w] < bi)) {
                bv = rv[w];
                bi = ri[w];
            }
        out_v[b] = bv;
        out_i[b] = bi == 0x7fffffff ? 0x7fffffff : bi + off;
    }
}

}  // namespace jdg

// jdg_hb1.cuh — batch-1 decode step of the host GGUF path (gguf_host_forward,
// janusdoe.c:3160-3322) as a chain of Programmatic-Dependent-Launch kernels over packed
// Q8_0 / Q4_K rows.
//
// Per layer (five launches):
//   QKV   x -> xn = rmsnorm(x, attn_norm) in every CTA's prologue; q|k|v = W . xn
//   ATTN  RoPE, KV append, per-chunk softmax partials (the own-model attention CTA), plus
//         CTAs that compute the 16 votes w_vote[e] . xn and the LoRA projections
//         t_e = B_e . xn of every alive expert (janusdoe.c:3281-3303 evaluate both on xn)
//   WO    merges the partials, x += Wo . att
//   GU    fn = rmsnorm(x, ffn_norm) in every CTA; h = silu(Wg . fn) * (Wu . fn); CTA 0 runs
//         the host election on the votes (janusdoe.c:3054-3087)
//   DN    x += focus * (Wd . h), then the LoRA deltas of the elected experts in election
//         order: x += (alpha * w_ki) * (A_e[i] . t_e)
// then LM (final RMSNorm prologue, logits, last-CTA greedy pick).
//
// Every kernel loads its first weight rows into registers before griddepcontrol.wait, so
// that HBM traffic overlaps the previous kernel.  Only data written two or more kernels
// back is read before a wait: DN finishes the LoRA dot products of every alive expert (t_e
// from ATTN) and reads its residual row (from WO) early, and the election (from GU, the
// kernel just before) after its wait.
#pragma once
#include "jdg_b1.cuh"
#include "jdg_host_kernels.cuh"

namespace jdg {

// One packed row in registers: this lane's 16-byte pieces of every 512-byte chunk of
// codes (Q8_0: 512 weights per chunk; Q4_K: 1024 weights), with their block scale
// (Q8_0: the f16 d of the lane's 32-weight block) or superblock header (Q4_K).
template <int DT, int MAXC>
struct PRow {
    uint4 q[MAXC];
    uint4 h[DT == 12 ? MAXC : 1];
    uint32_t s[DT == 8 ? MAXC : 1];
};

__device__ __forceinline__ uint32_t ld_nc_u16(const void *p) {
    unsigned short v;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ld_nc_u4(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

// chunks of 512 code bytes in a row of K weights
__host__ __device__ constexpr int prow_chunks(int dt, int K) { return dt == 8 ? (K + 511) / 512 : (K / 2 + 511) / 512; }

template <int DT, int MAXC>
__device__ __forceinline__ void prow_load(PRow<DT, MAXC> &r, const QW &w, int row, int lane) {
    const int K = w.cols;
    if (DT == 8) {
        const uint8_t *qr = w.q + (size_t)row * K;
        const uint16_t *sr = reinterpret_cast<const uint16_t *>(w.s) + (size_t)row * (K / 32);
#pragma unroll
        for (int j = 0; j < MAXC; j++) {
            const int e0 = lane * 16 + 512 * j;
            if (e0 < K) {
                r.q[j] = ld_stream_u4(qr + e0);
                r.s[j] = ld_nc_u16(sr + (e0 >> 5));
            }
        }
    } else {
        const uint8_t *qr = w.q + (size_t)row * (K / 2);
        const uint8_t *hr = w.s + (size_t)row * (K / 256) * 16;
#pragma unroll
        for (int j = 0; j < MAXC; j++) {
            const int b0 = lane * 16 + 512 * j;
            if (b0 < K / 2) {
                r.q[j] = ld_stream_u4(qr + b0);
                r.h[j] = ld_nc_u4(hr + (size_t)(b0 >> 7) * 16);
            }
        }
    }
}

// W[row] . x with the row in registers; the same per-lane arithmetic as qrow_dot.
// xsum: sums of 16 consecutive x (Q4_K min terms).
// Shared-memory layout of the vector a packed row multiplies: float4 L is stored at
// xsw(L), an XOR of its low bits, so that the 8 lanes of one 128-byte shared-memory phase hit
// 8 distinct 16-byte bank groups.  Q8_0 lanes read float4s 4*lane + c (+128 j); Q4_K lanes
// 8p+m read 64p + 16*(m/2) + 4*(m&1) + c.  The XOR stays inside aligned groups of 8 float4s.
template <int DT>
__device__ __forceinline__ int xsw(int L) { return DT == 8 ? (L ^ ((L >> 3) & 7)) : (L ^ ((L >> 4) & 3)); }
template <int DT>
__device__ __forceinline__ float4 xget4(const float *xs, int L) { return reinterpret_cast<const float4 *>(xs)[xsw<DT>(L)]; }
template <int DT>
__device__ __forceinline__ float xget(const float *xs, int e) { return xs[xsw<DT>(e >> 2) * 4 + (e & 3)]; }
template <int DT>
__device__ __forceinline__ void xput4(float *xs, int L, float4 v) { reinterpret_cast<float4 *>(xs)[xsw<DT>(L)] = v; }

// Exact code -> float conversion in two instructions per weight: PRMT places the code
// byte u under the exponent of 2^23 (bits 0x4B0000uu = 2^23 + u), FADD removes the offset.
// Q8_0 words are XORed with 0x80808080 first (u = q + 128).
__device__ __forceinline__ float byte_f(uint32_t w, int k, float off) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u + (unsigned)k)) - off;
}

// W[row] . x with the row in registers (the weight values of qrow_dot, janusdoe.c:2566-2585).
// xsum: sums of 16 consecutive x (Q4_K min terms).
template <int DT, int MAXC>
__device__ __forceinline__ float prow_dot(const PRow<DT, MAXC> &r, int K, const float *xs, const float *xsum, int lane) {
    float acc = 0.f;
    if (DT == 8) {
#pragma unroll
        for (int j = 0; j < MAXC; j++) {
            const int e0 = lane * 16 + 512 * j;
            if (e0 < K) {
                const float d = h2f((uint16_t)r.s[j]);
                const uint32_t wd[4] = {r.q[j].x ^ 0x80808080u, r.q[j].y ^ 0x80808080u, r.q[j].z ^ 0x80808080u,
                                        r.q[j].w ^ 0x80808080u};
                float s0 = 0.f, s1 = 0.f;
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const float4 xv = xget4<DT>(xs, (e0 >> 2) + c);
                    s0 = fmaf(byte_f(wd[c], 0, 8388736.0f), xv.x, s0);
                    s1 = fmaf(byte_f(wd[c], 1, 8388736.0f), xv.y, s1);
                    s0 = fmaf(byte_f(wd[c], 2, 8388736.0f), xv.z, s0);
                    s1 = fmaf(byte_f(wd[c], 3, 8388736.0f), xv.w, s1);
                }
                acc = fmaf(d, s0 + s1, acc);
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < MAXC; j++) {
            const int b0 = lane * 16 + 512 * j;
            if (b0 < K / 2) {
                const int sb = b0 >> 7, o = b0 & 127, c = o >> 5, l0 = o & 31;
                const uint8_t *hb = reinterpret_cast<const uint8_t *>(&r.h[j]);
                const float d = h2f((uint16_t)(hb[0] | (hb[1] << 8))), dmin = h2f((uint16_t)(hb[2] | (hb[3] << 8)));
                int s0, m0, s1, m1;
                smk4(2 * c, hb + 4, s0, m0);
                smk4(2 * c + 1, hb + 4, s1, m1);
                const float d1 = d * (float)s0, mm1 = dmin * (float)m0, d2 = d * (float)s1, mm2 = dmin * (float)m1;
                const int xb = sb * 256 + 64 * c + l0;
                const uint32_t wd[4] = {r.q[j].x, r.q[j].y, r.q[j].z, r.q[j].w};
                float sl = 0.f, sh = 0.f;
#pragma unroll
                for (int cc = 0; cc < 4; cc++) {
                    const float4 a4 = xget4<DT>(xs, (xb >> 2) + cc), b4 = xget4<DT>(xs, (xb >> 2) + 8 + cc);
                    const uint32_t lo = wd[cc] & 0x0F0F0F0Fu, hi = (wd[cc] >> 4) & 0x0F0F0F0Fu;
                    sl = fmaf(byte_f(lo, 0, 8388608.0f), a4.x, sl);
                    sh = fmaf(byte_f(hi, 0, 8388608.0f), b4.x, sh);
                    sl = fmaf(byte_f(lo, 1, 8388608.0f), a4.y, sl);
                    sh = fmaf(byte_f(hi, 1, 8388608.0f), b4.y, sh);
                    sl = fmaf(byte_f(lo, 2, 8388608.0f), a4.z, sl);
                    sh = fmaf(byte_f(hi, 2, 8388608.0f), b4.z, sh);
                    sl = fmaf(byte_f(lo, 3, 8388608.0f), a4.w, sl);
                    sh = fmaf(byte_f(hi, 3, 8388608.0f), b4.w, sh);
                }
                acc = fmaf(d1, sl, acc);
                acc = fmaf(-mm1, xsum[xb >> 4], acc);
                acc = fmaf(d2, sh, acc);
                acc = fmaf(-mm2, xsum[(xb + 32) >> 4], acc);
            }
        }
    }
    return warp_sum(acc);
}

struct HB1Args {
    int D, H, KVH, HD, qd, kd, qkvd, hidden, V, max_seq, L, R, l;
    float eps, lora_alpha, focus;
    QW w;                   // this kernel's matrix (q|k|v, Wo, gate/up interleaved, Wd, output)
    const float *norm;      // attn_norm / ffn_norm / output_norm (ones where the model has none)
    const float *tok_emb;
    const int *tok;
    int *pos;
    float *x, *xn, *y;      // residual, attention-normed input of the layer, output
    const float *hin;       // DN: the SwiGLU activations
    // LoRA parliament (janusdoe.c:3281-3303)
    const float *w_vote;    // [16][D]
    const float *lora_A;    // [16][D][R]
    const float *lora_B;    // [16][R][D]
    const int *alive;       // [16]
    const int *alive_list;  // alive expert ids in ascending order
    int n_alive;
    float *votes;           // [16]
    float *tall;            // [16][R]: t_e = B_e . xn for every alive e
    int *kcnt, *sel;
    float *selw, *consensus;
    int *tr_k, *tr_sel;
    float *tr_w, *tr_ema;
    // attention partials (merged by WO)
    const float *part;
    int natt;               // attention CTAs of the ATTN kernel
    // LM head pick
    unsigned *tickets;
    float *amax_v;
    int *amax_i;
    int *tok_out, *plen, *prompt, *hist, *hist_n, *next_out;
    int Hmax, greedy_pick;
    unsigned long long *stats;
    int *err;
    int embed;
    unsigned long long *tl;  // optional timeline [kernel][3] (engine debug)
};

// x (global) -> xs = x * inv * norm, with inv = 1/sqrt(mean(x^2) + eps) (janusdoe.c:3196-3199,
// 3230-3233); for Q4_K also the sums of 16.  Called by all 128 threads after the wait.
// Returns in xs; CTA 0 optionally stores the normalised vector.
template <int DT>
__device__ __forceinline__ void hb1_norm_x(const float *x, const float *norm, int D, float eps, float *xs, float *xsum,
                                           float *store, float *red) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < D / 4; i += 128) {
        const float4 v = __ldcg(reinterpret_cast<const float4 *>(x) + i);
        xput4<DT>(xs, i, v);
        ss = dot4(v, v, ss);
    }
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)D + eps);
    for (int i = threadIdx.x; i < D / 4; i += 128) {
        float4 v = xget4<DT>(xs, i);
        const float4 w = reinterpret_cast<const float4 *>(norm)[i];
        v.x = __fmul_rn(__fmul_rn(v.x, inv), w.x);
        v.y = __fmul_rn(__fmul_rn(v.y, inv), w.y);
        v.z = __fmul_rn(__fmul_rn(v.z, inv), w.z);
        v.w = __fmul_rn(__fmul_rn(v.w, inv), w.w);
        xput4<DT>(xs, i, v);
        if (store) reinterpret_cast<float4 *>(store)[i] = v;
    }
    __syncthreads();
    if (DT == 12) {
        for (int g = threadIdx.x; g < D / 16; g += 128) {
            float t = 0.f;
#pragma unroll
            for (int i = 0; i < 16; i++) t += xget<DT>(xs, 16 * g + i);
            xsum[g] = t;
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------------
// QKV: one row per warp.  Layer 0 gathers x = tok_emb[tok] (janusdoe.c:3191) first.
// Dynamic shared memory: D + D/16 floats.
template <int DT, int MAXC>
static __global__ __launch_bounds__(128) void k_hb1_qkv(HB1Args a) {
    TlMark tlm(a.tl, a.l * 5 + 0);
    extern __shared__ __align__(16) float hsm[];
    float *xs = hsm, *xsum = hsm + a.D;
    __shared__ float red[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row = blockIdx.x * 4 + warp;
    PRow<DT, MAXC> r;
    if (row < a.w.rows) prow_load<DT, MAXC>(r, a.w, row, lane);
    pdl_wait();
    tlm.waited();
    pdl_trigger();
    const float *xsrc = a.x;
    if (a.embed) {
        int t = a.tok[0];
        if (t < 0 || t >= a.V) {
            if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(a.err, JDG_ERR_TOKEN);
            t = 0;
        }
        xsrc = a.tok_emb + (size_t)t * a.D;
        if (blockIdx.x == 0)
            for (int i = threadIdx.x; i < a.D / 4; i += 128)
                reinterpret_cast<float4 *>(a.x)[i] = reinterpret_cast<const float4 *>(xsrc)[i];
    }
    hb1_norm_x<DT>(xsrc, a.norm, a.D, a.eps, xs, xsum, blockIdx.x == 0 ? a.xn : nullptr, red);
    if (row >= a.w.rows) return;
    const float v = prow_dot<DT, MAXC>(r, a.D, xs, xsum, lane);
    if (lane == 0) a.y[row] = v;
}

// ---------------------------------------------------------------------------------
// ATTN: CTAs [0, natt) are attention CTAs (chunk c = bid % nch, KV head g = bid / nch);
// the others compute one f32 row each per warp: rows 0..15 the votes w_vote[e] . xn
// (non-finite -> -1e30, janusdoe.c:3061), then R rows of B_e for every alive expert.
template <int HD>
static __global__ __launch_bounds__(128) void k_hb1_attn(B1Args ab, HB1Args a) {
    const int bid = blockIdx.x;
    TlMark tlm(a.tl, a.l * 5 + 1);
    if (bid < a.natt) {
        const int nch = a.natt / a.KVH;
        b1_attn_cta<HD>(ab, bid % nch, bid / nch, tlm);
        return;
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int arow = (bid - a.natt) * 4 + warp, nrows = kMaxE + a.n_alive * a.R;
    pdl_wait();
    tlm.waited();
    pdl_trigger();
    if (arow >= nrows) return;
    const float *wr;
    float *dst;
    bool vote = arow < kMaxE;
    if (vote) {
        wr = a.w_vote + (size_t)arow * a.D;
        dst = a.votes + arow;
    } else {
        const int j = arow - kMaxE, e = a.alive_list[j / a.R], rr = j % a.R;
        wr = a.lora_B + ((size_t)e * a.R + rr) * a.D;
        dst = a.tall + (size_t)e * a.R + rr;
    }
    float acc = 0.f;
    for (int k4 = lane; k4 < a.D / 4; k4 += 32)
        acc = dot4(ld_stream4(wr + 4 * k4), __ldcg(reinterpret_cast<const float4 *>(a.xn) + k4), acc);
    acc = warp_sum(acc);
    if (lane == 0) *dst = (vote && !isfinite(acc)) ? -1e30f : acc;
}

// The host election (janusdoe.c:3054-3087) on one thread: alive list ascending; na == 1
// takes that expert with weight 1 and leaves the EMA alone; top-k by strict '>' with the
// next unused alive expert when none beats -1e30; softmax without temperature, uniform
// weights when the sum is not finite and positive.  Every loop runs over the 16 expert
// slots unrolled with the alive mask (ascending order, the reference's operation order), so
// the votes, selection and weights stay in registers.
static __device__ void hb1_elect_serial(const HB1Args &a) {
    unsigned alive = 0;
    int na = 0, first = -1;
#pragma unroll
    for (int e = 0; e < kMaxE; e++)
        if (a.alive[e]) {
            alive |= 1u << e;
            if (first < 0) first = e;
            na++;
        }
    float *cons = a.consensus + a.l;
    int k = 0, sel[kMaxE];
    float w[kMaxE];
#pragma unroll
    for (int i = 0; i < kMaxE; i++) {
        sel[i] = -1;
        w[i] = 0.f;
    }
    if (na == 1) {
        k = 1;
        sel[0] = first;
        w[0] = 1.0f;
    } else if (na >= 2) {
        float v[kMaxE];
#pragma unroll
        for (int e = 0; e < kMaxE; e++) v[e] = __ldcg(a.votes + e);
        float mean = 0.f;
#pragma unroll
        for (int e = 0; e < kMaxE; e++)
            if (alive >> e & 1u) mean = __fadd_rn(mean, v[e]);
        mean = mean / (float)na;
        float var = 0.f;
#pragma unroll
        for (int e = 0; e < kMaxE; e++)
            if (alive >> e & 1u) {
                const float dd = __fsub_rn(v[e], mean);
                var = __fadd_rn(var, __fmul_rn(dd, dd));
            }
        var = var / (float)na;
        const float cs = fminf(1.0f, sqrtf(__fadd_rn(var, 1e-8f)) / __fadd_rn(fabsf(mean), 1.0f));
        const float ema = __fadd_rn(__fmul_rn(0.9f, *cons), __fmul_rn(0.1f, cs));
        *cons = ema;
        k = (int)__fmul_rn((float)na, __fsub_rn(1.0f, ema));
        if (k < 2) k = 2;
        if (k > na) k = na;
        unsigned used = 0;
#pragma unroll
        for (int ki = 0; ki < kMaxE; ki++) {
            if (ki < k) {
                float bv = -1e30f, bw = 0.f;
                int bi = -1;
#pragma unroll
                for (int e = 0; e < kMaxE; e++)
                    if ((alive & ~used) >> e & 1u && v[e] > bv) {
                        bv = v[e];
                        bi = e;
                    }
                if (bi < 0) bi = __ffs(alive & ~used) - 1;  // the next unused alive expert
#pragma unroll
                for (int e = 0; e < kMaxE; e++)
                    if (e == bi) bw = v[e];
                sel[ki] = bi;
                w[ki] = bw;
                used |= 1u << bi;
            }
        }
        float mx = w[0];
#pragma unroll
        for (int i = 1; i < kMaxE; i++)
            if (i < k && w[i] > mx) mx = w[i];
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < kMaxE; i++)
            if (i < k) {
                w[i] = expf(__fsub_rn(w[i], mx));
                sum = __fadd_rn(sum, w[i]);
            }
        const bool ok = sum > 0.0f && isfinite(sum);
#pragma unroll
        for (int i = 0; i < kMaxE; i++)
            if (i < k) w[i] = ok ? w[i] / sum : 1.0f / (float)k;
    }
    a.kcnt[0] = k;
    a.tr_k[a.l] = k;
    a.tr_ema[a.l] = *cons;
#pragma unroll
    for (int i = 0; i < kMaxE; i++) {
        a.sel[i] = i < k ? sel[i] : -1;
        a.selw[i] = i < k ? w[i] : 0.f;
        a.tr_sel[(size_t)a.l * kMaxE + i] = i < k ? sel[i] : -1;
        a.tr_w[(size_t)a.l * kMaxE + i] = i < k ? w[i] : 0.f;
    }
}

// ---------------------------------------------------------------------------------
// WO: att = merge of the attention partials; x[row] += Wo[row] . att (janusdoe.c:3226-3227).
// Dynamic smem: qd + qd/16 floats (att and, for Q4_K, its sums of 16).
template <int DT, int MAXC, int HD>
static __global__ __launch_bounds__(128) void k_hb1_wo(HB1Args a) {
    TlMark tlm(a.tl, a.l * 5 + 2);
    extern __shared__ __align__(16) float hsm[];
    constexpr int CH = kB1Chunk, MAXCH = 1024 / CH;
    __shared__ float fm[64][MAXCH];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row = blockIdx.x * 4 + warp;
    PRow<DT, MAXC> r;
    if (row < a.D) prow_load<DT, MAXC>(r, a.w, row, lane);
    const float xold = row < a.D ? __ldcg(a.x + row) : 0.f;
    const int p = __ldcg(a.pos), nc = p / CH + 1, ncs = a.max_seq / CH + 1;
    pdl_wait();
    tlm.waited();
    pdl_trigger();
    // merge weights per head: f_c = e^{m_c - M} / sum_c l_c e^{m_c - M}
    for (int h = threadIdx.x; h < a.H; h += 128) {
        float mv[MAXCH], lv[MAXCH], M = -INFINITY;
#pragma unroll
        for (int c = 0; c < MAXCH; c++) {
            const float *pp = a.part + ((size_t)h * ncs + c) * (HD + 2) + HD;
            mv[c] = c < nc ? __ldcg(pp) : -INFINITY;
            lv[c] = c < nc ? __ldcg(pp + 1) : 0.f;
            M = fmaxf(M, mv[c]);
        }
        float S = 0.f, f[MAXCH];
#pragma unroll
        for (int c = 0; c < MAXCH; c++) {
            f[c] = c < nc ? expf(mv[c] - M) : 0.f;
            S = fmaf(lv[c], f[c], S);
        }
#pragma unroll
        for (int c = 0; c < MAXCH; c++) fm[h][c] = f[c] / S;
    }
    __syncthreads();
#pragma unroll 2
    for (int i = threadIdx.x; i < a.qd; i += 128) {
        const int h = i / HD, d = i % HD;
        const float *pp = a.part + (size_t)h * ncs * (HD + 2) + d;
        float ov[MAXCH];  // every chunk's value loaded before the ordered sum
#pragma unroll
        for (int c = 0; c < MAXCH; c++) ov[c] = c < nc ? __ldcg(pp + (size_t)c * (HD + 2)) : 0.f;
        float o = 0.f;
#pragma unroll
        for (int c = 0; c < MAXCH; c++)
            if (c < nc) o = fmaf(ov[c], fm[h][c], o);
        hsm[xsw<DT>(i >> 2) * 4 + (i & 3)] = o;
    }
    __syncthreads();
    float *asum = hsm + a.qd;
    if (DT == 12) {
        for (int g = threadIdx.x; g < a.qd / 16; g += 128) {
            float t = 0.f;
#pragma unroll
            for (int i = 0; i < 16; i++) t += xget<DT>(hsm, 16 * g + i);
            asum[g] = t;
        }
        __syncthreads();
    }
    if (row >= a.D) return;
    const float v = prow_dot<DT, MAXC>(r, a.qd, hsm, asum, lane);
    if (lane == 0) a.x[row] = __fadd_rn(xold, v);
}

// ---------------------------------------------------------------------------------
// GU: fn = rmsnorm(x, ffn_norm) in every CTA, then units i (rows 2i gate, 2i+1 up of the
// interleaved matrix): h[i] = gate / (1 + expf(-gate)) * up (janusdoe.c:3236-3238).
// Persistent grid; warps stride over units with two units in flight; the first two load
// before the wait.  CTA 0 runs this layer's election instead: its votes were written two
// kernels back, so it starts at once and overlaps WO and GU.  Dynamic smem: D + D/16 floats.
template <int DT, int MAXC>
static __global__ __launch_bounds__(128) void k_hb1_gu(HB1Args a) {
    TlMark tlm(a.tl, a.l * 5 + 3);
    extern __shared__ __align__(16) float hsm[];
    float *xs = hsm, *xsum = hsm + a.D;
    __shared__ float red[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (blockIdx.x == 0) {
        if (threadIdx.x == 0) hb1_elect_serial(a);
        return;
    }
    const int nunits = a.w.rows / 2, gw = (gridDim.x - 1) * 4;
    PRow<DT, MAXC> ga, ua, gb, ub;
    int u = (blockIdx.x - 1) * 4 + warp;
    auto load_unit = [&](int uu, PRow<DT, MAXC> &g4, PRow<DT, MAXC> &u4) {
        if (uu >= nunits) return;
        prow_load<DT, MAXC>(g4, a.w, 2 * uu, lane);
        prow_load<DT, MAXC>(u4, a.w, 2 * uu + 1, lane);
    };
    auto compute_unit = [&](int uu, const PRow<DT, MAXC> &g4, const PRow<DT, MAXC> &u4) {
        const float g = prow_dot<DT, MAXC>(g4, a.D, xs, xsum, lane);
        const float v = prow_dot<DT, MAXC>(u4, a.D, xs, xsum, lane);
        if (lane == 0) a.y[uu] = __fmul_rn(silu_ref(g), v);
    };
    load_unit(u, ga, ua);
    load_unit(u + gw, gb, ub);
    pdl_wait();
    tlm.waited();
    pdl_trigger();
    hb1_norm_x<DT>(a.x, a.norm, a.D, a.eps, xs, xsum, nullptr, red);
    while (u < nunits) {
        compute_unit(u, ga, ua);
        load_unit(u + 2 * gw, ga, ua);
        u += gw;
        if (u >= nunits) break;
        compute_unit(u, gb, ub);
        load_unit(u + 2 * gw, gb, ub);
        u += gw;
    }
}

// ---------------------------------------------------------------------------------
// DN: x[row] += focus * (Wd[row] . h) (janusdoe.c:3239-3240), then for each elected expert
// in order x[row] += (alpha * w_ki) * (A_e[row] . t_e) (janusdoe.c:3293-3300).  The LoRA dot
// products of every alive expert use data two or more kernels old and finish before the
// wait; the election (GU) is read after it.  Dynamic smem: hidden + hidden/16 floats.
template <int DT, int MAXC>
static __global__ __launch_bounds__(128) void k_hb1_dn(HB1Args a) {
    TlMark tlm(a.tl, a.l * 5 + 4);
    extern __shared__ __align__(16) float hsm[];
    float *hs = hsm, *hsum = hsm + a.hidden;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row = blockIdx.x * 4 + warp;
    __shared__ float lo_s[4][kMaxE];
    PRow<DT, MAXC> r;
    if (row < a.D) prow_load<DT, MAXC>(r, a.w, row, lane);
    float xold = 0.f;
    if (row < a.D) {
        // t_e (ATTN) and this row of x (WO) are two or more kernels old: the LoRA dot
        // products A_e[row] . t_e of every alive expert finish before the wait
        xold = __ldcg(a.x + row);
        if (lane < a.n_alive) {
            const int e = a.alive_list[lane];
            const float *Ar = a.lora_A + ((size_t)e * a.D + row) * a.R;
            const float *tr = a.tall + (size_t)e * a.R;
            float lora = 0.f;
            for (int q = 0; q < a.R; q++) lora = fmaf(__ldg(Ar + q), __ldcg(tr + q), lora);
            lo_s[warp][e] = lora;
        }
    }
    pdl_wait();
    tlm.waited();
    pdl_trigger();
    // the election was made by GU, the kernel just before: read after the wait
    const int k = min(__ldcg(a.kcnt), kMaxE);
    int ek = 0;
    float wk = 0.f;
    if (lane < k) {
        ek = __ldcg(a.sel + lane);
        wk = __fmul_rn(a.lora_alpha, __ldcg(a.selw + lane));
        if (ek < 0 || ek >= kMaxE) {
            ek = 0;
            wk = 0.f;
        }
    }
    for (int i = threadIdx.x; i < a.hidden / 4; i += 128)
        xput4<DT>(hs, i, __ldcg(reinterpret_cast<const float4 *>(a.hin) + i));
    __syncthreads();
    if (DT == 12) {
        for (int g = threadIdx.x; g < a.hidden / 16; g += 128) {
            float t = 0.f;
#pragma unroll
            for (int i = 0; i < 16; i++) t += xget<DT>(hs, 16 * g + i);
            hsum[g] = t;
        }
        __syncthreads();
    }
    if (row >= a.D) return;
    const float v = prow_dot<DT, MAXC>(r, a.hidden, hs, hsum, lane);
    float xr = __fadd_rn(xold, __fmul_rn(v, a.focus));
    for (int ki = 0; ki < k; ki++) {
        const int e = __shfl_sync(JDG_FULL, ek, ki);
        const float w = __shfl_sync(JDG_FULL, wk, ki);
        xr = __fadd_rn(xr, __fmul_rn(w, lo_s[warp][e]));
    }
    if (lane == 0) a.x[row] = xr;
}

// ---------------------------------------------------------------------------------
// LM: logits = Wout . rmsnorm(x, output_norm) (janusdoe.c:3309-3321); per-CTA argmax
// partials; with greedy_pick the last CTA takes the first-index maximum or the prompt's
// next id and advances tok/pos/history (the pick of the own-model chain).  Persistent
// grid, two rows in flight per warp, the first two before the wait.  Dynamic smem:
// D + D/16 floats.
template <int DT, int MAXC>
static __global__ __launch_bounds__(128) void k_hb1_lm(HB1Args a) {
    TlMark tlm(a.tl, a.L * 5);
    extern __shared__ __align__(16) float hsm[];
    float *xs = hsm, *xsum = hsm + a.D;
    __shared__ float red[32];
    __shared__ float bv_s[4];
    __shared__ int bi_s[4];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int V = a.w.rows, gw = gridDim.x * 4;
    PRow<DT, MAXC> ra, rb;
    int row = blockIdx.x * 4 + warp;
    if (row < V) prow_load<DT, MAXC>(ra, a.w, row, lane);
    if (row + gw < V) prow_load<DT, MAXC>(rb, a.w, row + gw, lane);
    pdl_wait();
    tlm.waited();
    pdl_trigger();
    hb1_norm_x<DT>(a.x, a.norm, a.D, a.eps, xs, xsum, nullptr, red);
    float val = -INFINITY;
    int vi = 0x7fffffff;
    auto compute_row = [&](int rr, const PRow<DT, MAXC> &w4) {
        const float v = prow_dot<DT, MAXC>(w4, a.D, xs, xsum, lane);
        if (lane == 0) a.y[rr] = v;
        if (v > val) {  // rows visited in increasing order per warp: first max kept
            val = v;
            vi = rr;
        }
    };
    while (row < V) {
        compute_row(row, ra);
        if (row + 2 * gw < V) prow_load<DT, MAXC>(ra, a.w, row + 2 * gw, lane);
        row += gw;
        if (row >= V) break;
        compute_row(row, rb);
        if (row + 2 * gw < V) prow_load<DT, MAXC>(rb, a.w, row + 2 * gw, lane);
        row += gw;
    }
    if (lane == 0) {
        bv_s[warp] = val;
        bi_s[warp] = vi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float bv = bv_s[0];
        int bi = bi_s[0];
        for (int q = 1; q < 4; q++)
            if (bv_s[q] > bv || (bv_s[q] == bv && bi_s[q] < bi)) {
                bv = bv_s[q];
                bi = bi_s[q];
            }
        a.amax_v[blockIdx.x] = bv;
        a.amax_i[blockIdx.x] = bi;
    }
    if (!a.greedy_pick) return;
    if (!last_cta(a.tickets + 48, gridDim.x)) return;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int q = threadIdx.x; q < (int)gridDim.x; q += 128) {
        const float vv = __ldcg(a.amax_v + q);
        const int ii = __ldcg(a.amax_i + q);
        if (vv > bv || (vv == bv && ii < bi)) {
            bv = vv;
            bi = ii;
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
        for (int q = 1; q < 4; q++)
            if (bv_s[q] > bv_s[0] || (bv_s[q] == bv_s[0] && bi_s[q] < bi_s[0])) {
                bv_s[0] = bv_s[q];
                bi_s[0] = bi_s[q];
            }
        const int p = a.pos[0];
        atomicAdd(a.stats + 1, (unsigned long long)(p + 1));
        atomicAdd(a.stats + 2, 1ull);
        const bool from_prompt = a.plen && p + 1 < a.plen[0];
        const int nx = from_prompt ? a.prompt[p + 1] : (bi_s[0] == 0x7fffffff ? 0 : bi_s[0]);
        a.tok_out[0] = nx;
        a.pos[0] = p + 1;
        if (a.next_out) a.next_out[0] = nx;
        if (!from_prompt && a.hist) {
            const int hn = a.hist_n[0];
            if (hn < a.Hmax) a.hist[hn] = nx;
            a.hist_n[0] = hn + 1;
        }
        a.tickets[48] = 0;
    }
}

}  // namespace jdg

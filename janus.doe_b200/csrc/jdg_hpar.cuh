// jdg_hpar.cuh — batched host step around the tensor-core GEMM: the activation prep with
// the RMS norm folded in (one CTA per token), and the LoRA parliament of a layer
// (janusdoe.c:3281-3303) as two kernels over all sequences at once.
#pragma once
#include "jdg_qmma.cuh"

namespace jdg {

// ---------------------------------------------------------------------------------
// x -> (optionally RMS-normed, janusdoe.c:504 / 3196-3199) -> prepared activations of
// k_qm_q4k: the fp16 hi/lo rows t and 32 + t of every superblock's B tile (tensor-core K
// order) and row t of its B_min tile (the 8 sub-block sums, hi then lo along K).  grid 32: CTA t handles token slot t
// (slots >= M write zeros), block 256.  Norm: inv = 1/sqrt(mean(x^2) + eps) (each thread sums
// its 8-element groups in order, then the block), v = (x * inv) * w; norm_w null = ones.
// xn_out (optional) receives the normed rows.  Thread tid owns the groups g = tid + 256 m of
// 8 consecutive K positions (one 16-byte core-matrix row piece); a warp covers the 32 groups
// of one superblock, lanes 4j..4j+3 its sub-block j.  Loads go out in batches of 8 groups.
constexpr int kPrepBatch = 8;
static __global__ __launch_bounds__(256) void k_qm_prep_tok(const float *__restrict__ X, int ldx, int M, int K, int do_norm,
                                                            const float *__restrict__ norm_w, float eps,
                                                            float *__restrict__ xn_out, uint8_t *__restrict__ out) {
    __shared__ float red[32];
    // launched as a dependent of the previous kernel: wait for it before reading X; the GEMM
    // that follows (also a dependent launch) may start its weight stream now and waits for
    // this grid to finish before reading the prepared activations
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, ng = K / 8;
    const bool live = t < M;
    const float *xr = X + (size_t)t * ldx;
    float inv = 1.f;
    if (live && do_norm) {
        float ss = 0.f;
        for (int g0 = tid; g0 < ng; g0 += 256 * kPrepBatch) {
            float4 xa[kPrepBatch], xb[kPrepBatch];
#pragma unroll
            for (int m = 0; m < kPrepBatch; m++) {
                const int g = g0 + 256 * m;
                if (g < ng) {
                    xa[m] = *reinterpret_cast<const float4 *>(xr + 8 * g);
                    xb[m] = *reinterpret_cast<const float4 *>(xr + 8 * g + 4);
                }
            }
#pragma unroll
            for (int m = 0; m < kPrepBatch; m++)
                if (g0 + 256 * m < ng) {
                    ss = fmaf(xa[m].x, xa[m].x, ss); ss = fmaf(xa[m].y, xa[m].y, ss);
                    ss = fmaf(xa[m].z, xa[m].z, ss); ss = fmaf(xa[m].w, xa[m].w, ss);
                    ss = fmaf(xb[m].x, xb[m].x, ss); ss = fmaf(xb[m].y, xb[m].y, ss);
                    ss = fmaf(xb[m].z, xb[m].z, ss); ss = fmaf(xb[m].w, xb[m].w, ss);
                }
        }
        ss = block_sum(ss, red);
        inv = 1.0f / sqrtf(ss / (float)K + eps);
    }
    for (int g0 = tid; g0 < ng; g0 += 256 * kPrepBatch) {
        float4 xa[kPrepBatch], xb[kPrepBatch], wa[kPrepBatch], wb[kPrepBatch];
#pragma unroll
        for (int m = 0; m < kPrepBatch; m++) {
            const int g = g0 + 256 * m;
            xa[m] = xb[m] = make_float4(0.f, 0.f, 0.f, 0.f);
            wa[m] = wb[m] = make_float4(1.f, 1.f, 1.f, 1.f);
            if (live && g < ng) {
                xa[m] = *reinterpret_cast<const float4 *>(xr + 8 * g);
                xb[m] = *reinterpret_cast<const float4 *>(xr + 8 * g + 4);
                if (do_norm && norm_w) {
                    wa[m] = *reinterpret_cast<const float4 *>(norm_w + 8 * g);
                    wb[m] = *reinterpret_cast<const float4 *>(norm_w + 8 * g + 4);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < kPrepBatch; m++) {
            const int g = g0 + 256 * m;
            if (g >= ng) break;  // warp-uniform: ng is a multiple of 32
            const int sb = g / 32, c = g % 32;
            float v[8] = {xa[m].x, xa[m].y, xa[m].z, xa[m].w, xb[m].x, xb[m].y, xb[m].z, xb[m].w};
            if (live && do_norm) {
                const float w8[8] = {wa[m].x, wa[m].y, wa[m].z, wa[m].w, wb[m].x, wb[m].y, wb[m].z, wb[m].w};
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    v[i] = __fmul_rn(v[i], inv);
                    if (norm_w) v[i] = __fmul_rn(v[i], w8[i]);
                }
            }
            if (live && xn_out) {
                float *o = xn_out + (size_t)t * ldx + 8 * g;
                *reinterpret_cast<float4 *>(o) = make_float4(v[0], v[1], v[2], v[3]);
                *reinterpret_cast<float4 *>(o + 4) = make_float4(v[4], v[5], v[6], v[7]);
            }
            uint8_t *tile = out + (size_t)sb * kQmBBytes;
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float a0 = v[qm_kperm(2 * i)], a1 = v[qm_kperm(2 * i + 1)];
                hi[i] = qm_split2(a0, a1, false);
                lo[i] = qm_split2(a0, a1, true);
            }
            *reinterpret_cast<uint4 *>(tile + ((size_t)(c * (kQmN / 8) + t / 8) * 8 + t % 8) * 16) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            const int tl = kQmTok + t;
            *reinterpret_cast<uint4 *>(tile + ((size_t)(c * (kQmN / 8) + tl / 8) * 8 + tl % 8) * 16) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            // sub-block sums: 8 values here, then the 4 lanes of the sub-block
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < 8; i++) s += v[i];
            s += __shfl_xor_sync(JDG_FULL, s, 1);
            s += __shfl_xor_sync(JDG_FULL, s, 2);
            float sj[8];
#pragma unroll
            for (int j = 0; j < 8; j++) sj[j] = __shfl_sync(JDG_FULL, s, 4 * j);
            if (lane == 0) {
                uint8_t *bm = tile + kQmBMain;
                uint32_t h[4], l[4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    h[i] = qm_split2(sj[2 * i], sj[2 * i + 1], false);
                    l[i] = qm_split2(sj[2 * i], sj[2 * i + 1], true);
                }
                // B_min row t: K columns 0..7 the hi parts, 8..15 the lo parts
                *reinterpret_cast<uint4 *>(bm + ((size_t)(0 * (kQmTok / 8) + t / 8) * 8 + t % 8) * 16) = make_uint4(h[0], h[1], h[2], h[3]);
                *reinterpret_cast<uint4 *>(bm + ((size_t)(1 * (kQmTok / 8) + t / 8) * 8 + t % 8) * 16) = make_uint4(l[0], l[1], l[2], l[3]);
            }
        }
    }
}

// ---------------------------------------------------------------------------------
// LoRA parliament of one layer for B sequences (janusdoe.c:3281-3303).
struct HParArgs {
    int D, R, B, L, l;
    const float *xn;        // [B][D] attention-normed layer input
    const float *w_vote;    // [16][D]
    const float *lora_A;    // [16][D][R]
    const float *lora_B;    // [16][R][D]
    const int *alive;       // [16]
    const int *alive_list;  // alive expert ids, ascending
    int n_alive;
    float *part;            // [D/256][n_alive][R+1][B] partial dots
    unsigned *tickets;      // [n_alive + 1], zero between launches
    float *votes;           // [B][16]
    float *tall;            // [B][16][R]: t = B_e . xn for every alive e
    int *kcnt, *sel;
    float *selw, *consensus;
    int *tr_k, *tr_sel;
    float *tr_w, *tr_ema;
    float lora_alpha;
    float *x;               // [B][D] residual
};
constexpr int kHparTok = 32;   // sequences per k_hpar_dots launch
constexpr int kHparXs = 260;   // padded row of the staged activations (conflict-free float4 reads)
// dynamic shared memory of k_hpar_dots: 32 activation rows and R + 1 (<= 24) weight rows of 256
__host__ __device__ constexpr size_t hpar_dots_smem(int R) { return ((size_t)kHparTok * kHparXs + (size_t)(R + 1) * 256) * 4; }

// Votes w_vote[e] . xn[b] and LoRA-B projections B_e[r] . xn[b] of every alive expert for all
// sequences.  grid (D/256, n_alive), block 256, dynamic smem hpar_dots_smem(R) (R + 1 <= 24):
// CTA (kc, ei) takes the 256-wide K chunk kc of the R+1 rows of expert alive_list[ei] for all
// B (<= 32) sequences and stores partial dots; the last CTA of an expert (ticket) adds its
// chunks in order, the last expert to finish runs the B elections (host_parliament_elect
// rules, one thread per sequence).
static __global__ __launch_bounds__(256) void k_hpar_dots(HParArgs a) {
    extern __shared__ __align__(16) float hsm_dots[];
    float(*xs)[kHparXs] = reinterpret_cast<float(*)[kHparXs]>(hsm_dots);
    float(*ws)[256] = reinterpret_cast<float(*)[256]>(hsm_dots + kHparTok * kHparXs);
    __shared__ unsigned s_last;
    const int kc = blockIdx.x, ei = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int e = a.alive_list[ei], R = a.R, nrow = R + 1, k0 = kc * 256;
    {
        // every load of the staging issued before the first store (B <= 32: 8 float4 of
        // activations per thread; R + 1 <= 21: 6 float4 of weight rows)
        float4 xv[8], wv[6];
#pragma unroll
        for (int m = 0; m < 8; m++) {
            const int i = tid + 256 * m, b = i / 64, q = i % 64;
            if (i < a.B * 64) xv[m] = *reinterpret_cast<const float4 *>(a.xn + (size_t)b * a.D + k0 + 4 * q);
        }
#pragma unroll
        for (int m = 0; m < 6; m++) {
            const int i = tid + 256 * m, r = i / 64, q = i % 64;
            if (i < nrow * 64) {
                const float *src = r == 0 ? a.w_vote + (size_t)e * a.D : a.lora_B + ((size_t)e * R + (r - 1)) * a.D;
                wv[m] = *reinterpret_cast<const float4 *>(src + k0 + 4 * q);
            }
        }
#pragma unroll
        for (int m = 0; m < 8; m++) {
            const int i = tid + 256 * m;
            if (i < a.B * 64) *reinterpret_cast<float4 *>(&xs[i / 64][4 * (i % 64)]) = xv[m];
        }
#pragma unroll
        for (int m = 0; m < 6; m++) {
            const int i = tid + 256 * m;
            if (i < nrow * 64) *reinterpret_cast<float4 *>(&ws[i / 64][4 * (i % 64)]) = wv[m];
        }
    }
    __syncthreads();
    // lane = sequence, warp w takes rows w, w + 8, w + 16
    float acc[3] = {0.f, 0.f, 0.f};
    if (lane < a.B) {
        for (int q = 0; q < 64; q++) {
            const float4 xv = *reinterpret_cast<const float4 *>(&xs[lane][4 * q]);
#pragma unroll
            for (int m = 0; m < 3; m++) {
                const int r = warp + 8 * m;
                if (r < nrow) acc[m] = dot4(*reinterpret_cast<const float4 *>(&ws[r][4 * q]), xv, acc[m]);
            }
        }
#pragma unroll
        for (int m = 0; m < 3; m++) {
            const int r = warp + 8 * m;
            if (r < nrow) a.part[(((size_t)kc * a.n_alive + ei) * nrow + r) * kHparTok + lane] = acc[m];
        }
    }
    // the last K chunk of this expert adds the chunks in order
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        s_last = atomicAdd(a.tickets + ei, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int nkc = gridDim.x;
    for (int i = tid; i < nrow * a.B; i += 256) {
        const int r = i / a.B, b = i % a.B;
        float s = 0.f;
        for (int c0 = 0; c0 < nkc; c0 += 16) {  // chunks in order, sixteen loads in flight
            float v[16];
#pragma unroll
            for (int m = 0; m < 16; m++)
                v[m] = c0 + m < nkc ? __ldcg(a.part + (((size_t)(c0 + m) * a.n_alive + ei) * nrow + r) * kHparTok + b) : 0.f;
#pragma unroll
            for (int m = 0; m < 16; m++)
                if (c0 + m < nkc) s += v[m];
        }
        if (r == 0) a.votes[b * kMaxE + e] = isfinite(s) ? s : -1e30f;
        else a.tall[((size_t)b * kMaxE + e) * R + (r - 1)] = s;
    }
    __syncthreads();
    if (tid == 0) {
        a.tickets[ei] = 0;
        __threadfence();
        s_last = atomicAdd(a.tickets + a.n_alive, 1u) == (unsigned)a.n_alive - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (tid == 0) a.tickets[a.n_alive] = 0;
    if (tid < a.B) {
        // one sequence's election through the batch-1 routine, with its rows of every array
        HB1Args h = {};
        h.l = a.l;
        h.alive = a.alive;
        h.votes = a.votes + tid * kMaxE;
        h.consensus = a.consensus + (size_t)tid * a.L;
        h.kcnt = a.kcnt + tid;
        h.sel = a.sel + tid * kMaxE;
        h.selw = a.selw + tid * kMaxE;
        h.tr_k = a.tr_k + (size_t)tid * a.L;
        h.tr_ema = a.tr_ema + (size_t)tid * a.L;
        h.tr_sel = a.tr_sel + (size_t)tid * a.L * kMaxE;
        h.tr_w = a.tr_w + (size_t)tid * a.L * kMaxE;
        hb1_elect_serial(h);
    }
}

// x[b][i] += (alpha * w_ki) * (A_e[i] . t_e[b]) for the elected experts in election order
// (janusdoe.c:3294-3302).  grid (D/32), block 256, dynamic smem hpar_apply_smem: CTA takes rows
// i0..i0+31 of every alive expert's A (rows padded to R + 4 floats: the 8 lanes of a
// shared-memory phase read 8 consecutive rows from 8 distinct bank groups) and the
// projections t of all sequences into shared memory; thread (b, q) updates rows i0+q+8m
// (m < 4) of sequence b (B <= 32, R % 4 == 0).
__host__ __device__ constexpr size_t hpar_apply_smem(int n_alive, int R) {
    return ((size_t)n_alive * 32 * (R + 4) + (size_t)kHparTok * n_alive * R) * 4;
}
static __global__ __launch_bounds__(256) void k_hpar_apply(HParArgs a) {
    extern __shared__ __align__(16) float hsm_apply[];
    const int R = a.R, na = a.n_alive;
    const int RP = R + 4;                      // padded row of A
    float *as = hsm_apply;                     // [na][32][RP]
    float *ts = hsm_apply + (size_t)na * 32 * RP;  // [32][na][R]
    __shared__ int slot[kMaxE];                // expert id -> index in alive_list
    __shared__ int s_sel[kHparTok][kMaxE], s_k[kHparTok];
    __shared__ float s_w[kHparTok][kMaxE];
    const int i0 = blockIdx.x * 32, tid = threadIdx.x;
    if (tid < kMaxE) slot[tid] = -1;
    {
        // the elections of all sequences (2 entries per thread, loads before stores)
        int sv[2] = {-1, -1}, kv = 0;
        float wv[2] = {0.f, 0.f};
#pragma unroll
        for (int m = 0; m < 2; m++) {
            const int i = tid + 256 * m;
            if (i < a.B * kMaxE) {
                sv[m] = a.sel[i];
                wv[m] = a.selw[i];
            }
        }
        if (tid < a.B) kv = a.kcnt[tid];
#pragma unroll
        for (int m = 0; m < 2; m++) {
            const int i = tid + 256 * m;
            if (i < a.B * kMaxE) {
                s_sel[i / kMaxE][i % kMaxE] = sv[m];
                s_w[i / kMaxE][i % kMaxE] = wv[m];
            }
        }
        if (tid < a.B) s_k[tid] = kv;
    }
    __syncthreads();
    if (tid < na) slot[a.alive_list[tid]] = tid;
    // staging in float4 units, eight loads in flight per thread before their stores
    const int nA = na * 8 * R, nT = a.B * na * (R / 4);
    for (int base = 0; base < nA + nT; base += 256 * 8) {
        float4 v[8];
#pragma unroll
        for (int m = 0; m < 8; m++) {
            const int idx = base + tid + 256 * m;
            if (idx < nA) {
                const int ei = idx / (8 * R), rem = idx % (8 * R);
                if (i0 + (4 * rem) / R < a.D)
                    v[m] = *reinterpret_cast<const float4 *>(a.lora_A + ((size_t)a.alive_list[ei] * a.D + i0) * R + 4 * rem);
            } else if (idx < nA + nT) {
                const int j = idx - nA, b = j / (na * (R / 4)), rem = j % (na * (R / 4)), ei = rem / (R / 4), q = rem % (R / 4);
                v[m] = __ldcg(reinterpret_cast<const float4 *>(a.tall + ((size_t)b * kMaxE + a.alive_list[ei]) * R) + q);
            }
        }
#pragma unroll
        for (int m = 0; m < 8; m++) {
            const int idx = base + tid + 256 * m;
            if (idx < nA) {
                const int ei = idx / (8 * R), rem = idx % (8 * R), row = (4 * rem) / R, col = (4 * rem) % R;
                if (i0 + row < a.D) *reinterpret_cast<float4 *>(as + ((size_t)ei * 32 + row) * RP + col) = v[m];
            } else if (idx < nA + nT) {
                reinterpret_cast<float4 *>(ts)[idx - nA] = v[m];
            }
        }
    }
    __syncthreads();
    const int b = tid >> 3, q = tid & 7;
    if (b >= a.B) return;
    float xi[4];
#pragma unroll
    for (int m = 0; m < 4; m++) {
        const int i = i0 + q + 8 * m;
        xi[m] = i < a.D ? a.x[(size_t)b * a.D + i] : 0.f;
    }
    const int k = s_k[b];
    for (int ki = 0; ki < k; ki++) {
        const int e = s_sel[b][ki], si = (e >= 0 && e < kMaxE) ? slot[e] : -1;
        if (si < 0) continue;  // the election only picks alive experts
        const float w = __fmul_rn(a.lora_alpha, s_w[b][ki]);
        const float *tr = ts + ((size_t)b * na + si) * R;
        float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
        for (int r = 0; r < R; r += 4) {
            const float4 tv = *reinterpret_cast<const float4 *>(tr + r);
#pragma unroll
            for (int m = 0; m < 4; m++) {
                const float4 av = *reinterpret_cast<const float4 *>(as + ((size_t)si * 32 + q + 8 * m) * RP + r);
                s[m] = fmaf(av.x, tv.x, s[m]);
                s[m] = fmaf(av.y, tv.y, s[m]);
                s[m] = fmaf(av.z, tv.z, s[m]);
                s[m] = fmaf(av.w, tv.w, s[m]);
            }
        }
#pragma unroll
        for (int m = 0; m < 4; m++) xi[m] = __fadd_rn(xi[m], __fmul_rn(w, s[m]));
    }
#pragma unroll
    for (int m = 0; m < 4; m++) {
        const int i = i0 + q + 8 * m;
        if (i < a.D) a.x[(size_t)b * a.D + i] = xi[m];
    }
}

}  // namespace jdg

// jdg_kernels.cuh — decode-step kernels for the own model and the shared pieces of the
// host path: embedding, RMSNorm, f32 GEMV (batch <= 8), f32 SIMT GEMM (grouped by expert),
// RoPE + KV append, split-K decode attention, the parliament election, routing, expert
// combine, and next-token selection.  Every kernel cites the reference lines it replaces.
#pragma once
#include "jdg_async.cuh"
#include "jdg_common.cuh"

namespace jdg {

constexpr int kMaxE = 16;
constexpr int kAttnChunk = 64;  // positions per attention CTA (k_attn_partial)
constexpr int kAttnRowsChunk = 32;  // positions per attention CTA (k_attn_rows)
constexpr int kMaxHG = 8;       // query heads per KV head supported by the attention kernel

// ------------------------------------------------------------------------------------
// x[b] = tok_emb[tok[b]] (janusdoe.c:882; host janusdoe.c:3177 zero row for token >= V)
static __global__ void k_embed(const float *__restrict__ emb, int V, int D, const int *__restrict__ tok, float *__restrict__ x,
                        int *err) {
    int b = blockIdx.x, t = tok[b];
    float *xr = x + (size_t)b * D;
    if (t < 0 || t >= V) {
        if (threadIdx.x == 0) atomicOr(err, JDG_ERR_TOKEN);
        for (int i = threadIdx.x; i < D; i += blockDim.x) xr[i] = 0.f;
        return;
    }
    const float *er = emb + (size_t)t * D;
    for (int i = threadIdx.x; i < D; i += blockDim.x) xr[i] = er[i];
}

// out[b] = x[b] * (1/sqrtf(sum(x^2)/D + eps)) * w   (janusdoe.c:504, 3181-3186); w may be null
// 1 / sqrt(mean(x^2) + eps) of one row, the whole block taking part (janusdoe.c:504): thread
// t sums elements t, t + blockDim, ... in order with eight loads in flight, then block_sum.
__device__ __forceinline__ float rms_inv(const float *__restrict__ xr, int D, float eps, float *red) {
    float ss = 0.f;
    for (int base = 0; base < D; base += blockDim.x * 8) {
        float v[8];
#pragma unroll
        for (int m = 0; m < 8; m++) {
            const int i = base + threadIdx.x + blockDim.x * m;
            v[m] = i < D ? xr[i] : 0.f;
        }
#pragma unroll
        for (int m = 0; m < 8; m++)
            if (base + threadIdx.x + blockDim.x * m < D) ss = fmaf(v[m], v[m], ss);
    }
    ss = block_sum(ss, red);
    return 1.0f / sqrtf(ss / (float)D + eps);
}
static __global__ void k_rmsnorm(const float *__restrict__ x, const float *__restrict__ w, float *__restrict__ out, int D,
                          float eps) {
    __shared__ float red[32];
    int b = blockIdx.x;
    const float *xr = x + (size_t)b * D;
    const float inv = rms_inv(xr, D, eps, red);
    float *o = out + (size_t)b * D;
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        float v = __fmul_rn(xr[i], inv);
        o[i] = w ? __fmul_rn(v, w[i]) : v;
    }
}

// ------------------------------------------------------------------------------------
// f32 GEMV for NB <= 8 tokens: Y[b][row] (epi) W[row][:] . X[b][:]  (matvec, janusdoe.c:505-519)
// One warp per RPW rows, X staged in shared memory, optionally RMS-normalised on the way in.
enum { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2 };

struct GemvArgs {
    const float *W;
    int N, K;
    const float *X;
    int ldx;
    const float *norm_w;  // prenorm weights (nullptr with prenorm = ones)
    float eps;
    int prenorm;
    float *Y;
    int ldy;
};

template <int NB, int RPW, int EPI>
static __global__ __launch_bounds__(128) void k_gemv_f32(GemvArgs a) {
    extern __shared__ float xs[];  // [NB][K]
    __shared__ float red[32];
    const int K = a.K, K4 = K >> 2;
    for (int b = 0; b < NB; b++) {
        const float4 *src = reinterpret_cast<const float4 *>(a.X + (size_t)b * a.ldx);
        float4 *dst = reinterpret_cast<float4 *>(xs + (size_t)b * K);
        float ss = 0.f;
        for (int i = threadIdx.x; i < K4; i += blockDim.x) {
            float4 v = src[i];
            dst[i] = v;
            ss = dot4(v, v, ss);
        }
        if (a.prenorm) {
            ss = block_sum(ss, red);
            float inv = 1.0f / sqrtf(ss / (float)K + a.eps);
            for (int i = threadIdx.x; i < K; i += blockDim.x) {
                float v = __fmul_rn(xs[b * K + i], inv);
                xs[b * K + i] = a.norm_w ? __fmul_rn(v, a.norm_w[i]) : v;
            }
        }
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row0 = (blockIdx.x * (blockDim.x >> 5) + warp) * RPW;
    if (row0 >= a.N) return;
    float acc[RPW][NB];
#pragma unroll
    for (int r = 0; r < RPW; r++)
#pragma unroll
        for (int b = 0; b < NB; b++) acc[r][b] = 0.f;
    const float *wr[RPW];
#pragma unroll
    for (int r = 0; r < RPW; r++) wr[r] = a.W + (size_t)min(row0 + r, a.N - 1) * K;
    const float4 *xs4 = reinterpret_cast<const float4 *>(xs);
#pragma unroll 4
    for (int k4 = lane; k4 < K4; k4 += 32) {
        float4 w[RPW];
#pragma unroll
        for (int r = 0; r < RPW; r++) w[r] = ld_stream4(wr[r] + 4 * k4);
#pragma unroll
        for (int b = 0; b < NB; b++) {
            float4 xv = xs4[b * K4 + k4];
#pragma unroll
            for (int r = 0; r < RPW; r++) acc[r][b] = dot4(w[r], xv, acc[r][b]);
        }
    }
#pragma unroll
    for (int r = 0; r < RPW; r++)
#pragma unroll
        for (int b = 0; b < NB; b++) acc[r][b] = warp_sum(acc[r][b]);
    if (lane != 0) return;
#pragma unroll
    for (int b = 0; b < NB; b++) {
        float *y = a.Y + (size_t)b * a.ldy;
        if (EPI == EPI_SWIGLU) {
            // rows (2i, 2i+1) = (gate_i, up_i): h_i = silu(g)*u  (janusdoe.c:925)
            y[row0 >> 1] = __fmul_rn(silu_ref(acc[0][b]), acc[RPW - 1][b]);
        } else {
#pragma unroll
            for (int r = 0; r < RPW; r++) {
                int row = row0 + r;
                if (row < a.N) {
                    if (EPI == EPI_ADD) y[row] = __fadd_rn(y[row], acc[r][b]);
                    else y[row] = acc[r][b];
                }
            }
        }
    }
}

// ------------------------------------------------------------------------------------
// Expert FFN for one token (janusdoe.c:921-929): gate/up of each elected expert.
// grid (ceil(2H / (4 warps * 2 rows)), 16): y = election slot ki; rows 2i/2i+1 = gate_i/up_i.
static __global__ __launch_bounds__(128) void k_expert_gu_b1(const float *const *__restrict__ gu_tab, const int *__restrict__ kcnt,
                                                      const int *__restrict__ sel, int H, int D,
                                                      const float *__restrict__ xb, float *__restrict__ hbuf, int *err) {
    extern __shared__ float xs[];
    const int ki = blockIdx.y;
    if (ki >= kcnt[0]) return;
    const int e = sel[ki];
    if (e < 0 || e >= kMaxE || gu_tab[e] == nullptr) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(err, JDG_ERR_ROUTE);
        return;
    }
    const float *W = gu_tab[e];
    const int K4 = D >> 2;
    for (int i = threadIdx.x; i < K4; i += blockDim.x) reinterpret_cast<float4 *>(xs)[i] = reinterpret_cast<const float4 *>(xb)[i];
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int i = blockIdx.x * (blockDim.x >> 5) + warp;  // hidden unit
    if (i >= H) return;
    const float *wg = W + (size_t)(2 * i) * D, *wu = wg + D;
    float ag = 0.f, au = 0.f;
    const float4 *xs4 = reinterpret_cast<const float4 *>(xs);
#pragma unroll 4
    for (int k4 = lane; k4 < K4; k4 += 32) {
        float4 g = ld_stream4(wg + 4 * k4), u = ld_stream4(wu + 4 * k4), xv = xs4[k4];
        ag = dot4(g, xv, ag);
        au = dot4(u, xv, au);
    }
    ag = warp_sum(ag);
    au = warp_sum(au);
    if (lane == 0) hbuf[(size_t)ki * H + i] = __fmul_rn(silu_ref(ag), au);
}

// Down projection of every elected expert for one token, then the weighted sum in election
// order and the residual add: expert_out += w_ki * (Wd_e . h_ki); x += expert_out
// (janusdoe.c:926-929).  grid ceil(D / 4 warps).
static __global__ __launch_bounds__(128) void k_expert_down_b1(const float *const *__restrict__ dn_tab, const int *__restrict__ kcnt,
                                                        const int *__restrict__ sel, const float *__restrict__ selw, int D, int H,
                                                        const float *__restrict__ hbuf, float *__restrict__ x) {
    extern __shared__ float hs[];  // [k][H]
    const int k = kcnt[0];
    const int H4 = H >> 2;
    for (int i = threadIdx.x; i < k * H4; i += blockDim.x) reinterpret_cast<float4 *>(hs)[i] = reinterpret_cast<const float4 *>(hbuf)[i];
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r = blockIdx.x * (blockDim.x >> 5) + warp;
    if (r >= D) return;
    float eo = 0.f;
    for (int ki = 0; ki < k; ki++) {
        const float *W = dn_tab[sel[ki]];
        if (W == nullptr) continue;
        const float *wr = W + (size_t)r * H;
        const float4 *h4 = reinterpret_cast<const float4 *>(hs + (size_t)ki * H);
        float acc = 0.f;
#pragma unroll 4
        for (int k4 = lane; k4 < H4; k4 += 32) acc = dot4(ld_stream4(wr + 4 * k4), h4[k4], acc);
        acc = warp_sum(acc);
        eo = __fadd_rn(eo, __fmul_rn(selw[ki], acc));
    }
    if (lane == 0) x[r] = __fadd_rn(x[r], eo);
}

// ------------------------------------------------------------------------------------
// f32 SIMT GEMM, optionally grouped by expert: C[row(m)][n] (epi) sum_k A[arow(m)][k] * W[n][k]
// Tile BM x 128 x 16, 256 threads, thread tile (BM/16) x 8, register double buffering.
struct SgemmArgs {
    const float *A;
    int lda;
    const int *idx;   // grouped + gathered: A row of (segment s, m) = idx[s*ldi + m]
    int ldi;
    int a_seg_rows;   // grouped, not gathered: A row = s*a_seg_rows + m
    const int *cnt;   // grouped: rows of segment s = cnt[s]; nullptr = dense with M rows
    int M;
    const float *const *Wtab;  // grouped: weights of segment s
    const float *W;
    int N, K;
    float *C;
    int ldc;
    int c_seg_rows;   // grouped: C row = s*c_seg_rows + m
};

template <int BM, int EPI>
static __global__ __launch_bounds__(256) void k_sgemm(SgemmArgs a) {
    constexpr int BN = 128, BK = 16, TM = BM / 16;
    const int seg = blockIdx.z;
    const int M = a.cnt ? a.cnt[seg] : a.M;
    const int m0 = blockIdx.y * BM;
    if (m0 >= M) return;
    const float *W = a.Wtab ? a.Wtab[seg] : a.W;
    if (W == nullptr) return;
    const int n0 = blockIdx.x * BN;
    const int tid = threadIdx.x;
    __shared__ __align__(16) float As[2][BK][BM + 4];
    __shared__ __align__(16) float Ws[2][BK][BN + 4];

    // loader mapping
    const int la_row = tid >> 2, la_k4 = tid & 3;  // A: BM rows x 4 float4
    const bool la_on = la_row < BM;
    const float *a_src = nullptr;
    if (la_on && m0 + la_row < M) {
        int m = m0 + la_row, ar;
        if (a.cnt && a.idx) ar = a.idx[seg * a.ldi + m];
        else if (a.cnt) ar = seg * a.a_seg_rows + m;
        else ar = m;
        a_src = a.A + (size_t)ar * a.lda;
    }
    const float *w_src[2];
#pragma unroll
    for (int j = 0; j < 2; j++) {
        int n = n0 + la_row + 64 * j;
        w_src[j] = n < a.N ? W + (size_t)n * a.K : nullptr;
    }
    float4 ra, rw[2];
    auto gload = [&](int k0) {
        ra = a_src ? *reinterpret_cast<const float4 *>(a_src + k0 + 4 * la_k4) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 2; j++)
            rw[j] = w_src[j] ? ld_stream4(w_src[j] + k0 + 4 * la_k4) : make_float4(0.f, 0.f, 0.f, 0.f);
    };
    auto sstore = [&](int buf) {
        if (la_on) {
            As[buf][4 * la_k4 + 0][la_row] = ra.x;
            As[buf][4 * la_k4 + 1][la_row] = ra.y;
            As[buf][4 * la_k4 + 2][la_row] = ra.z;
            As[buf][4 * la_k4 + 3][la_row] = ra.w;
        }
#pragma unroll
        for (int j = 0; j < 2; j++) {
            int n = la_row + 64 * j;
            Ws[buf][4 * la_k4 + 0][n] = rw[j].x;
            Ws[buf][4 * la_k4 + 1][n] = rw[j].y;
            Ws[buf][4 * la_k4 + 2][n] = rw[j].z;
            Ws[buf][4 * la_k4 + 3][n] = rw[j].w;
        }
    };
    const int ty = tid >> 4, tx = tid & 15;
    float acc[TM][8];
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.f;

    const int nk = a.K / BK;
    gload(0);
    sstore(0);
    __syncthreads();
    for (int kt = 0; kt < nk; kt++) {
        const int buf = kt & 1;
        if (kt + 1 < nk) gload((kt + 1) * BK);
#pragma unroll
        for (int kk = 0; kk < BK; kk++) {
            float av[TM];
#pragma unroll
            for (int i = 0; i < TM; i++) av[i] = As[buf][kk][ty * TM + i];
            float4 w0 = *reinterpret_cast<const float4 *>(&Ws[buf][kk][tx * 4]);
            float4 w1 = *reinterpret_cast<const float4 *>(&Ws[buf][kk][64 + tx * 4]);
            float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = fmaf(av[i], wv[j], acc[i][j]);
        }
        if (kt + 1 < nk) sstore(buf ^ 1);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < TM; i++) {
        int m = m0 + ty * TM + i;
        if (m >= M) continue;
        size_t crow = a.cnt ? (size_t)seg * a.c_seg_rows + m : (size_t)m;
        float *c = a.C + crow * a.ldc;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            int nb = n0 + 64 * h + tx * 4;
            if (EPI == EPI_SWIGLU) {
#pragma unroll
                for (int p = 0; p < 4; p += 2)
                    if (nb + p + 1 < a.N) c[(nb + p) >> 1] = __fmul_rn(silu_ref(acc[i][4 * h + p]), acc[i][4 * h + p + 1]);
            } else {
#pragma unroll
                for (int p = 0; p < 4; p++) {
                    int n = nb + p;
                    if (n < a.N) {
                        if (EPI == EPI_ADD) c[n] = __fadd_rn(c[n], acc[i][4 * h + p]);
                        else c[n] = acc[i][4 * h + p];
                    }
                }
            }
        }
    }
}

// ------------------------------------------------------------------------------------
// RoPE on q and k heads of the fused qkv row, then append k and v to the cache at pos.
// Own model: NeoX-half pairs from the alloc_run cache (janusdoe.c:536, 864-873, 893-897).
// Host: NORM (2i,2i+1) or NEOX pairs (janusdoe.c:3198-3224).
// Element (token t, column n) of the product: the ks partials loaded first, then added in
// split order from zero (the arithmetic of the reduce kernel).
__device__ __forceinline__ float split_sum(const SplitPart &sp, int t, int n) {
    constexpr int kMaxSplitSum = kSplitMax;
    const size_t tile = (size_t)(t / kSplitTile) * sp.rtiles + n / kSplitTile;
    const float *p = sp.part + (tile * sp.ks * kSplitTile + t % kSplitTile) * kSplitTile + n % kSplitTile;
    float v[kMaxSplitSum];
#pragma unroll
    for (int z = 0; z < kMaxSplitSum; z++) v[z] = z < sp.ks ? __ldcg(p + (size_t)z * kSplitTile * kSplitTile) : 0.f;
    float s = 0.f;
#pragma unroll
    for (int z = 0; z < kMaxSplitSum; z++)
        if (z < sp.ks) s = __fadd_rn(s, v[z]);
    return s;
}

struct RopeArgs {
    float *qkv;
    int ld;          // row stride of qkv
    int H, KVH, HD;
    const float *cos_t, *sin_t;  // [max_seq][HD/2]
    int pair_norm;
    const int *pos;
    int max_seq;
    float *kc, *vc;  // layer base; slot b at + b*bstride, position t at + t*kd
    long bstride;
    int *err;
    SplitPart sp;  // when set, q/k/v are summed from the product's split-K partials here
};
static __global__ void k_rope_kv(RopeArgs a) {
    const int b = blockIdx.x, p = a.pos[b];
    if (p < 0 || p >= a.max_seq) {
        if (threadIdx.x == 0) atomicOr(a.err, JDG_ERR_POS);
        return;
    }
    const int half = a.HD >> 1, kd = a.KVH * a.HD, qd = a.H * a.HD;
    float *row = a.qkv + (size_t)b * a.ld;
    const float *ct = a.cos_t + (size_t)p * half, *st = a.sin_t + (size_t)p * half;
    float *kdst = a.kc + (size_t)b * a.bstride + (size_t)p * kd;
    float *vdst = a.vc + (size_t)b * a.bstride + (size_t)p * kd;
    const int npair = (a.H + a.KVH) * half;
    for (int idx = threadIdx.x; idx < npair; idx += blockDim.x) {
        int h = idx / half, i = idx - h * half;
        int i0 = a.pair_norm ? 2 * i : i, i1 = a.pair_norm ? 2 * i + 1 : i + half;
        float *v = row + (size_t)h * a.HD;  // q heads then k heads are contiguous
        float x0, x1;
        if (a.sp.part) {
            x0 = split_sum(a.sp, b, h * a.HD + i0);
            x1 = split_sum(a.sp, b, h * a.HD + i1);
        } else {
            x0 = v[i0];
            x1 = v[i1];
        }
        const float c = ct[i], s = st[i];
        float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        float y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        if (h < a.H) {
            v[i0] = y0;
            v[i1] = y1;
        } else {
            int kh = h - a.H;
            kdst[kh * a.HD + i0] = y0;
            kdst[kh * a.HD + i1] = y1;
        }
    }
    const float *vsrc = row + qd + kd;
    for (int i = threadIdx.x; i < kd; i += blockDim.x) vdst[i] = a.sp.part ? split_sum(a.sp, b, qd + kd + i) : vsrc[i];
}

// ------------------------------------------------------------------------------------
// Decode attention over t <= pos, split into chunks of 64 positions (flash-decoding):
// s_t = (q.k_t)*scale*bias, clamp*tanh(s/clamp) when clamp > 0 (janusdoe.c:899-910, own
// model), no clamp for host (janusdoe.c:3226-3252); softmax; o = sum a_t v_t.  Each CTA
// writes (unnormalised o, chunk max, chunk sum) per head; k_attn_combine merges chunks.
struct AttnArgs {
    const float *qkv;
    int ld;
    const float *kc, *vc;
    long bstride;
    const int *pos;
    int H, KVH, HD, hg, nchunk;
    float scale, bias, clamp, inv_clamp;
    float *part;  // [B][H][nchunk][HD+2]
};
template <int HD>
static __global__ __launch_bounds__(128) void k_attn_partial(AttnArgs a) {
    constexpr int E = HD / 32;  // dims per lane
    const int c = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int p = a.pos[b], t0 = c * kAttnChunk;
    if (t0 > p) return;
    const int nt = min(kAttnChunk, p + 1 - t0);
    const int kd = a.KVH * HD, hg = a.hg;
    __shared__ __align__(16) float q_s[kMaxHG][HD];
    __shared__ float s_s[kMaxHG][kAttnChunk];
    __shared__ __align__(16) float o_s[4][kMaxHG][HD];
    const float *qrow = a.qkv + (size_t)b * a.ld + (size_t)g * hg * HD;
    for (int i = threadIdx.x; i < hg * HD; i += blockDim.x) q_s[i / HD][i % HD] = qrow[i];
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float *kbase = a.kc + (size_t)b * a.bstride + (size_t)t0 * kd + (size_t)g * HD;
    const float *vbase = a.vc + (size_t)b * a.bstride + (size_t)t0 * kd + (size_t)g * HD;
    for (int t = warp; t < nt; t += 4) {
        const float *kr = kbase + (size_t)t * kd + lane * E;
        float kv[E];
#pragma unroll
        for (int e = 0; e < E; e++) kv[e] = kr[e];
        for (int j = 0; j < hg; j++) {
            float d = 0.f;
#pragma unroll
            for (int e = 0; e < E; e++) d = fmaf(q_s[j][lane * E + e], kv[e], d);
            d = warp_sum(d);
            if (lane == 0) {
                float s = __fmul_rn(d, a.scale);
                if (a.bias != 1.0f) s = __fmul_rn(s, a.bias);
                if (a.clamp > 0.f) s = __fmul_rn(a.clamp, tanhf(__fmul_rn(s, a.inv_clamp)));
                s_s[j][t] = s;
            }
        }
    }
    __syncthreads();
    __shared__ float m_s[kMaxHG], l_s[kMaxHG];
    for (int j = warp; j < hg; j += 4) {
        float m = -INFINITY;
        for (int t = lane; t < nt; t += 32) m = fmaxf(m, s_s[j][t]);
        m = warp_max(m);
        float l = 0.f;
        for (int t = lane; t < nt; t += 32) {
            float e = expf(s_s[j][t] - m);
            s_s[j][t] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) {
            m_s[j] = m;
            l_s[j] = l;
        }
    }
    __syncthreads();
    float o[kMaxHG][E];
#pragma unroll
    for (int j = 0; j < kMaxHG; j++)
#pragma unroll
        for (int e = 0; e < E; e++) o[j][e] = 0.f;
    for (int t = warp; t < nt; t += 4) {
        const float *vr = vbase + (size_t)t * kd + lane * E;
        float vv[E];
#pragma unroll
        for (int e = 0; e < E; e++) vv[e] = vr[e];
#pragma unroll
        for (int j = 0; j < kMaxHG; j++) {
            if (j < hg) {
                float pj = s_s[j][t];
#pragma unroll
                for (int e = 0; e < E; e++) o[j][e] = fmaf(pj, vv[e], o[j][e]);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < kMaxHG; j++)
        if (j < hg)
#pragma unroll
            for (int e = 0; e < E; e++) o_s[warp][j][lane * E + e] = o[j][e];
    __syncthreads();
    for (int i = threadIdx.x; i < hg * HD; i += blockDim.x) {
        int j = i / HD, d = i % HD;
        float v = o_s[0][j][d] + o_s[1][j][d] + o_s[2][j][d] + o_s[3][j][d];
        int h = g * hg + j;
        float *dst = a.part + (((size_t)b * a.H + h) * a.nchunk + c) * (HD + 2);
        dst[d] = v;
        if (d == 0) {
            dst[HD] = m_s[j];
            dst[HD + 1] = l_s[j];
        }
    }
}

// merge chunk partials: o = sum_c o_c e^{m_c-M} / sum_c l_c e^{m_c-M}; grid (H, B), block HD
// Decode attention, one CTA per (chunk of 32 positions, row) over every head: the chunk's
// key and value rows (all KV heads, contiguous in the cache) are copied to shared memory with
// 16-byte cp.async (rows padded by 4 floats so that lanes reading different rows hit
// different banks), then warp h scores its query head against position t = lane (one
// sequential fmaf chain over the head dimension), takes the chunk's max and sum in the warp,
// and lane d accumulates sum_t p_t v_t[d] in position order.  Same (o, max, sum) partials as
// k_attn_partial.  Block = H * 32 threads; dynamic shared memory attn_rows_smem().
__host__ __device__ inline size_t attn_rows_smem(int H, int HD, int kd) {
    return ((size_t)2 * kAttnRowsChunk * (kd + 4) + (size_t)H * HD + (size_t)H * kAttnRowsChunk) * 4;
}
template <int HD>
static __global__ __launch_bounds__(1024) void k_attn_rows(AttnArgs a) {
    constexpr int E = HD / 32;
    extern __shared__ __align__(16) float ar_sm[];
    const int c = blockIdx.x, b = blockIdx.y;
    const int p = a.pos[b], t0 = c * kAttnRowsChunk;
    if (t0 > p) return;
    const int nt = min(kAttnRowsChunk, p + 1 - t0);
    const int kd = a.KVH * HD, ks = kd + 4;
    float *k_s = ar_sm, *v_s = k_s + (size_t)kAttnRowsChunk * ks, *q_s = v_s + (size_t)kAttnRowsChunk * ks;
    float *p_s = q_s + a.H * HD;
    const int tid = threadIdx.x, nthr = blockDim.x;
    {
        const float *ksrc = a.kc + (size_t)b * a.bstride + (size_t)t0 * kd;
        const float *vsrc = a.vc + (size_t)b * a.bstride + (size_t)t0 * kd;
        const int q4 = kd / 4, n4 = nt * q4;
        for (int i = tid; i < n4; i += nthr) {
            const int t = i / q4, d = (i % q4) * 4;
            const uint32_t dk = smem_u32(k_s + t * ks + d), dv = smem_u32(v_s + t * ks + d);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dk), "l"(ksrc + (size_t)t * kd + d) : "memory");
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dv), "l"(vsrc + (size_t)t * kd + d) : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        const float *qrow = a.qkv + (size_t)b * a.ld;
        for (int i = tid; i < a.H * HD; i += nthr) q_s[i] = qrow[i];
        asm volatile("cp.async.wait_all;" ::: "memory");
    }
    __syncthreads();
    const int h = tid >> 5, lane = tid & 31, g = h / a.hg;
    float s = -INFINITY;
    if (lane < nt) {
        const float *kr = k_s + lane * ks + g * HD, *qh = q_s + h * HD;
        float d = 0.f;
#pragma unroll
        for (int i = 0; i < HD; i += 4) {
            const float4 kv = *reinterpret_cast<const float4 *>(kr + i);
            const float4 qv = *reinterpret_cast<const float4 *>(qh + i);
            d = fmaf(qv.x, kv.x, d);
            d = fmaf(qv.y, kv.y, d);
            d = fmaf(qv.z, kv.z, d);
            d = fmaf(qv.w, kv.w, d);
        }
        s = __fmul_rn(d, a.scale);
        if (a.bias != 1.0f) s = __fmul_rn(s, a.bias);
        if (a.clamp > 0.f) s = __fmul_rn(a.clamp, tanhf(__fmul_rn(s, a.inv_clamp)));
    }
    const float m = warp_max(s);
    const float ex = lane < nt ? expf(s - m) : 0.f;
    const float l = warp_sum(ex);
    p_s[h * kAttnRowsChunk + lane] = ex;
    __syncwarp();
    float o[E];
#pragma unroll
    for (int e = 0; e < E; e++) o[e] = 0.f;
    const float *vcol = v_s + g * HD + lane * E;
    for (int t = 0; t < nt; t++) {
        const float pt = p_s[h * kAttnRowsChunk + t];
#pragma unroll
        for (int e = 0; e < E; e++) o[e] = fmaf(pt, vcol[(size_t)t * ks + e], o[e]);
    }
    float *dst = a.part + (((size_t)b * a.H + h) * a.nchunk + c) * (HD + 2);
#pragma unroll
    for (int e = 0; e < E; e++) dst[lane * E + e] = o[e];
    if (lane == 0) {
        dst[HD] = m;
        dst[HD + 1] = l;
    }
}

// Merge of the chunk partials of one (row, head): o[d] = sum_c o_c[d] f_c / sum_c l_c f_c with
// f_c = e^{m_c - M}, in chunk order.  The chunks' (m, l) pairs are staged in shared memory
// (ml: 2 * nc floats) by the whole block first, so no load waits on another.
__device__ __forceinline__ float attn_merge(const float *__restrict__ pp, int nc, int HD, int d, float *ml) {
    for (int c = threadIdx.x; c < nc; c += blockDim.x) {
        ml[2 * c] = pp[(size_t)c * (HD + 2) + HD];
        ml[2 * c + 1] = pp[(size_t)c * (HD + 2) + HD + 1];
    }
    __syncthreads();
    float M = -INFINITY;
    for (int c = 0; c < nc; c++) M = fmaxf(M, ml[2 * c]);
    float S = 0.f, o = 0.f;
#pragma unroll 8
    for (int c = 0; c < nc; c++) {
        const float f = expf(ml[2 * c] - M);
        S = fmaf(ml[2 * c + 1], f, S);
        o = fmaf(pp[(size_t)c * (HD + 2) + d], f, o);
    }
    return o / S;
}
// grid (H, rows), block HD, dynamic shared memory 2 * nchunk floats
static __global__ void k_attn_combine(const float *__restrict__ part, const int *__restrict__ pos, int H, int HD, int nchunk,
                               int chunk, float *__restrict__ out, int ldo) {
    extern __shared__ float ac_ml[];
    const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    const int nc = pos[b] / chunk + 1;
    const float o = attn_merge(part + ((size_t)b * H + h) * nchunk * (HD + 2), nc, HD, d, ac_ml);
    out[(size_t)b * ldo + h * HD + d] = o;
}

// ------------------------------------------------------------------------------------
// Parliament election, one CTA per sequence (janusdoe.c:779-838 own; janusdoe.c:3054-3087
// host).  Own: xb = rmsnorm(x, ffn_norm) first (janusdoe.c:915) and the votes read xb.
// Host: the votes read the attention-norm output xn.  Votes are fp32 dots; the scalar
// election (mean, var, consensus EMA, variable k, strict-> top-k, softmax) runs on one
// thread in the reference's order.  The harmonic term is 0 during decode.
struct ElectArgs {
    const float *x;        // own: residual (normed here); host: xn (used as is)
    const float *norm_w;   // own: ffn_norm
    float eps;
    int D;
    int host;              // 1 = host_parliament_elect rules
    const float *w_vote;   // [16][D]
    const int *alive;      // [16]
    float temperature;
    float *consensus;      // [B][L]
    int L, l;
    float *xb;             // own: normed output [B][D]
    int *kcnt;             // [B]
    int *sel;              // [B][16]
    float *selw;           // [B][16]
    int *tr_k, *tr_sel;
    float *tr_w, *tr_ema;  // [B][L](*16)
    // prompt prefill (own model): rows are the tokens of one sequence; k_elect only writes
    // each token's votes and consensus measure, k_elect_scan runs the EMA over the tokens
    int prefill;
    float *pf_votes;       // [B][16]
    float *pf_cs;          // [B]
    float *pf_cons;        // the sequence's EMA of this layer (in: before the prompt, out: after)
    // own model only: when sp is set, the residual is x + (Wo product summed from its split-K
    // partials), written back to x_out before the norm
    SplitPart sp;
    float *x_out;
};

// The selection half of parliament_elect (janusdoe.c:811-837) / host_parliament_elect
// (janusdoe.c:3067-3085) from the votes v[e] of the alive slots and the updated EMA.
__device__ __forceinline__ int elect_select(const float *v, const int *alive_idx, int na, float ema, int host,
                                            float temperature, int *sel, float *w) {
    int k = (int)__fmul_rn((float)na, __fsub_rn(1.0f, ema));
    if (k < 2) k = 2;
    if (k > na) k = na;
    bool used[kMaxE];
    for (int e = 0; e < kMaxE; e++) used[e] = false;
    for (int ki = 0; ki < k; ki++) {
        float bv = -1e30f;
        int bi = host ? -1 : 0;
        for (int i = 0; i < na; i++) {
            const int e = alive_idx[i];
            if (!used[e] && v[e] > bv) {
                bv = v[e];
                bi = e;
            }
        }
        if (bi < 0)
            for (int i = 0; i < na; i++)
                if (!used[alive_idx[i]]) {
                    bi = alive_idx[i];
                    break;
                }
        sel[ki] = bi;
        w[ki] = v[bi];
        used[bi] = true;
    }
    const float temp = host ? 1.0f : (temperature > 0.05f ? temperature : 1.0f);
    float mx = w[0];
    for (int i = 1; i < k; i++)
        if (w[i] > mx) mx = w[i];
    float sum = 0.f;
    for (int i = 0; i < k; i++) {
        float arg = __fsub_rn(w[i], mx);
        if (!host) arg = arg / temp;
        w[i] = expf(arg);
        sum = __fadd_rn(sum, w[i]);
    }
    if (!host || (sum > 0.0f && isfinite(sum))) {
        for (int i = 0; i < k; i++) w[i] = w[i] / sum;
    } else {
        for (int i = 0; i < k; i++) w[i] = 1.0f / (float)k;
    }
    return k;
}

// consensus measure of one election: fminf(1, std / (|mean| + 1)) over the alive votes
__device__ __forceinline__ float elect_cs(const float *v, const int *alive_idx, int na) {
    float mean = 0.f;
    for (int i = 0; i < na; i++) mean = __fadd_rn(mean, v[alive_idx[i]]);
    mean = mean / (float)na;
    float var = 0.f;
    for (int i = 0; i < na; i++) {
        const float dd = __fsub_rn(v[alive_idx[i]], mean);
        var = __fadd_rn(var, __fmul_rn(dd, dd));
    }
    var = var / (float)na;
    return fminf(1.0f, sqrtf(__fadd_rn(var, 1e-8f)) / __fadd_rn(fabsf(mean), 1.0f));
}

static __global__ __launch_bounds__(256) void k_elect(ElectArgs a) {
    extern __shared__ float xs[];
    __shared__ float red[32];
    __shared__ float votes[kMaxE];
    const int b = blockIdx.x, D = a.D;
    const float *xr = a.x + (size_t)b * D;
    if (!a.host && a.sp.part) {
        // x + Wo.att from the split-K partials (the reduce kernel's sum and residual add),
        // kept in xs; elements tid, tid + blockDim, ... in order, four at a time
        float ss = 0.f;
        for (int base = 0; base < D; base += blockDim.x * 4) {
            float xo[4], pv[4];
#pragma unroll
            for (int m = 0; m < 4; m++) {
                const int i = base + threadIdx.x + blockDim.x * m;
                xo[m] = i < D ? xr[i] : 0.f;
                pv[m] = i < D ? split_sum(a.sp, b, i) : 0.f;
            }
#pragma unroll
            for (int m = 0; m < 4; m++) {
                const int i = base + threadIdx.x + blockDim.x * m;
                if (i < D) {
                    const float xn = __fadd_rn(xo[m], pv[m]);
                    a.x_out[(size_t)b * D + i] = xn;
                    xs[i] = xn;
                    ss = fmaf(xn, xn, ss);
                }
            }
        }
        ss = block_sum(ss, red);
        const float inv = 1.0f / sqrtf(ss / (float)D + a.eps);
        for (int i = threadIdx.x; i < D; i += blockDim.x) {
            const float v = __fmul_rn(__fmul_rn(xs[i], inv), a.norm_w[i]);
            xs[i] = v;
            a.xb[(size_t)b * D + i] = v;
        }
    } else if (!a.host) {
        // elements tid, tid + blockDim, ... in order, eight loads in flight
        float ss = 0.f;
        for (int base = 0; base < D; base += blockDim.x * 8) {
            float v[8];
#pragma unroll
            for (int m = 0; m < 8; m++) {
                const int i = base + threadIdx.x + blockDim.x * m;
                v[m] = i < D ? xr[i] : 0.f;
            }
#pragma unroll
            for (int m = 0; m < 8; m++)
                if (base + threadIdx.x + blockDim.x * m < D) ss = fmaf(v[m], v[m], ss);
        }
        ss = block_sum(ss, red);
        float inv = 1.0f / sqrtf(ss / (float)D + a.eps);
        for (int i = threadIdx.x; i < D; i += blockDim.x) {
            float v = __fmul_rn(__fmul_rn(xr[i], inv), a.norm_w[i]);
            xs[i] = v;
            a.xb[(size_t)b * D + i] = v;
        }
    } else {
        for (int i = threadIdx.x; i < D; i += blockDim.x) xs[i] = xr[i];
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int e = warp; e < kMaxE; e += nw) {
        if (!a.alive[e]) continue;
        const float *wr = a.w_vote + (size_t)e * D;
        float d = 0.f;
        for (int base = 0; base < D; base += 32 * 8) {  // in order, eight loads in flight
            float v[8];
#pragma unroll
            for (int m = 0; m < 8; m++) {
                const int i = base + lane + 32 * m;
                v[m] = i < D ? wr[i] : 0.f;
            }
#pragma unroll
            for (int m = 0; m < 8; m++) {
                const int i = base + lane + 32 * m;
                if (i < D) d = fmaf(v[m], xs[i], d);
            }
        }
        d = warp_sum(d);
        if (lane == 0) votes[e] = d;
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    int alive_idx[kMaxE], na = 0;
    for (int e = 0; e < kMaxE; e++)
        if (a.alive[e]) alive_idx[na++] = e;
    if (a.prefill) {  // votes and the consensus measure only; the EMA is a scan over the prompt
        for (int e = 0; e < kMaxE; e++) a.pf_votes[(size_t)b * kMaxE + e] = a.alive[e] ? votes[e] : 0.f;
        a.pf_cs[b] = na >= 2 ? elect_cs(votes, alive_idx, na) : 0.f;
        return;
    }
    float *cons = a.consensus + (size_t)b * a.L + a.l;
    int k = 0;
    int sel[kMaxE];
    float w[kMaxE];
    if (a.host && na == 1) {
        k = 1;
        sel[0] = alive_idx[0];
        w[0] = 1.0f;
    } else if ((!a.host && na >= 2) || (a.host && na >= 2)) {
        float v[kMaxE];
        for (int i = 0; i < na; i++) {
            int e = alive_idx[i];
            float d = votes[e];
            if (a.host && !isfinite(d)) d = -1e30f;
            v[e] = d;  // own: dot + 0.1f * 0 (harmonic state is zero at decode)
        }
        float mean = 0.f;
        for (int i = 0; i < na; i++) mean = __fadd_rn(mean, v[alive_idx[i]]);
        mean = mean / (float)na;
        float var = 0.f;
        for (int i = 0; i < na; i++) {
            float dd = __fsub_rn(v[alive_idx[i]], mean);
            var = __fadd_rn(var, __fmul_rn(dd, dd));
        }
        var = var / (float)na;
        float cs = fminf(1.0f, sqrtf(__fadd_rn(var, 1e-8f)) / __fadd_rn(fabsf(mean), 1.0f));
        float ema = __fadd_rn(__fmul_rn(0.9f, *cons), __fmul_rn(0.1f, cs));
        *cons = ema;
        k = (int)__fmul_rn((float)na, __fsub_rn(1.0f, ema));
        if (k < 2) k = 2;
        if (k > na) k = na;
        bool used[kMaxE];
        for (int e = 0; e < kMaxE; e++) used[e] = false;
        for (int ki = 0; ki < k; ki++) {
            float bv = -1e30f;
            int bi = a.host ? -1 : 0;
            for (int i = 0; i < na; i++) {
                int e = alive_idx[i];
                if (!used[e] && v[e] > bv) {
                    bv = v[e];
                    bi = e;
                }
            }
            if (bi < 0)
                for (int i = 0; i < na; i++)
                    if (!used[alive_idx[i]]) {
                        bi = alive_idx[i];
                        break;
                    }
            sel[ki] = bi;
            w[ki] = v[bi];
            used[bi] = true;
        }
        float temp = a.host ? 1.0f : (a.temperature > 0.05f ? a.temperature : 1.0f);
        float mx = w[0];
        for (int i = 1; i < k; i++)
            if (w[i] > mx) mx = w[i];
        float sum = 0.f;
        for (int i = 0; i < k; i++) {
            float arg = __fsub_rn(w[i], mx);
            if (!a.host) arg = arg / temp;
            w[i] = expf(arg);
            sum = __fadd_rn(sum, w[i]);
        }
        if (!a.host || (sum > 0.0f && isfinite(sum))) {
            for (int i = 0; i < k; i++) w[i] = w[i] / sum;
        } else {
            for (int i = 0; i < k; i++) w[i] = 1.0f / (float)k;
        }
    }
    a.kcnt[b] = k;
    for (int i = 0; i < kMaxE; i++) {
        a.sel[b * kMaxE + i] = i < k ? sel[i] : -1;
        a.selw[b * kMaxE + i] = i < k ? w[i] : 0.f;
    }
    size_t tl = (size_t)b * a.L + a.l;
    a.tr_k[tl] = k;
    a.tr_ema[tl] = *cons;
    for (int i = 0; i < kMaxE; i++) {
        a.tr_sel[tl * kMaxE + i] = i < k ? sel[i] : -1;
        a.tr_w[tl * kMaxE + i] = i < k ? w[i] : 0.f;
    }
}

// Prompt prefill: the EMA of one layer over the B prompt tokens in order
// (c_t = 0.9 c_{t-1} + 0.1 cs_t, the recurrence parliament_elect applies token by token,
// janusdoe.c:809), then every token's election from its own EMA value in parallel.
static __global__ __launch_bounds__(256) void k_elect_scan(ElectArgs a, int B) {
    extern __shared__ float ema_t[];  // [B]
    __shared__ int alive_idx[kMaxE], na_s;
    if (threadIdx.x == 0) {
        int na = 0;
        for (int e = 0; e < kMaxE; e++)
            if (a.alive[e]) alive_idx[na++] = e;
        na_s = na;
        float c = *a.pf_cons;
        if (na >= 2)
            for (int t = 0; t < B; t++) {
                c = __fadd_rn(__fmul_rn(0.9f, c), __fmul_rn(0.1f, a.pf_cs[t]));
                ema_t[t] = c;
            }
        else
            for (int t = 0; t < B; t++) ema_t[t] = c;
        *a.pf_cons = c;
    }
    __syncthreads();
    const int na = na_s;
    for (int t = threadIdx.x; t < B; t += blockDim.x) {
        int sel[kMaxE];
        float w[kMaxE], v[kMaxE];
        for (int e = 0; e < kMaxE; e++) v[e] = a.pf_votes[(size_t)t * kMaxE + e];
        const int k = na >= 2 ? elect_select(v, alive_idx, na, ema_t[t], 0, a.temperature, sel, w) : 0;
        a.kcnt[t] = k;
        const size_t tl = (size_t)t * a.L + a.l;
        a.tr_k[tl] = k;
        a.tr_ema[tl] = ema_t[t];
        for (int i = 0; i < kMaxE; i++) {
            a.sel[t * kMaxE + i] = i < k ? sel[i] : -1;
            a.selw[t * kMaxE + i] = i < k ? w[i] : 0.f;
            a.tr_sel[tl * kMaxE + i] = i < k ? sel[i] : -1;
            a.tr_w[tl * kMaxE + i] = i < k ? w[i] : 0.f;
        }
    }
}

// x[i] += y[i] * s (the residual add of a scaled FFN output)
static __global__ void k_add_scaled(float *x, const float *y, float s, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = __fadd_rn(x[i], __fmul_rn(y[i], s));
}

// ------------------------------------------------------------------------------------
// Bucket (sequence, election slot) pairs by expert, in ascending sequence order.
// grid 1, block 512 (warp e = expert slot).  idx[e*B + j] = b; pairrow[b*16+ki] = e*B + j.
// The elections of up to 512 sequences are first staged in shared memory (one byte per
// slot, 0xFF past kcnt), so every warp scans them without global-memory round trips.
static __global__ __launch_bounds__(512) void k_route(const int *__restrict__ kcnt, const int *__restrict__ sel, int B,
                                               int *__restrict__ cnt, int *__restrict__ idx, int *__restrict__ pairrow,
                                               unsigned long long *stats) {
    static_assert(kMaxE == 16, "one 16-byte row of slots per sequence");
    __shared__ __align__(16) uint8_t sel_s[512][kMaxE];
    const int e = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int n = 0;
    for (int base = 0; base < B; base += 512) {
        const int nb = min(512, B - base);
        __syncthreads();
        for (int i = threadIdx.x; i < nb * kMaxE; i += 512) {
            const int b = i / kMaxE, s = i % kMaxE;
            sel_s[b][s] = s < kcnt[base + b] ? (uint8_t)sel[(size_t)(base + b) * kMaxE + s] : (uint8_t)0xFF;
        }
        __syncthreads();
        for (int b0 = 0; b0 < nb; b0 += 32) {
            const int bl = b0 + lane;
            int ki = -1;
            if (bl < nb) {
                const uint4 w = *reinterpret_cast<const uint4 *>(sel_s[bl]);
                const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int i = 0; i < kMaxE; i++)
                    if (((words[i >> 2] >> (8 * (i & 3))) & 0xFFu) == (uint32_t)e) ki = i;
            }
            const unsigned m = __ballot_sync(JDG_FULL, ki >= 0);
            if (ki >= 0) {
                const int j = n + __popc(m & ((1u << lane) - 1)), b = base + bl;
                idx[e * B + j] = b;
                pairrow[b * kMaxE + ki] = e * B + j;
            }
            n += __popc(m);
        }
    }
    if (lane == 0) {
        cnt[e] = n;
        if (n > 0) atomicAdd(stats, 1ull);
    }
}

// x[b] += sum_ki w[b][ki] * y[pairrow(b,ki)] in election order (janusdoe.c:927-929)
// (the sequence's weights and rows are staged in shared memory, then every expert output of a
// column is loaded before the sum)
static __global__ void k_combine(const int *__restrict__ kcnt, const float *__restrict__ selw, const int *__restrict__ pairrow,
                          const float *__restrict__ y, int D, float *__restrict__ x) {
    __shared__ float w_s[kMaxE];
    __shared__ int row_s[kMaxE];
    const int b = blockIdx.x, k = kcnt[b];
    if (threadIdx.x < kMaxE) {
        w_s[threadIdx.x] = threadIdx.x < k ? selw[b * kMaxE + threadIdx.x] : 0.f;
        row_s[threadIdx.x] = threadIdx.x < k ? pairrow[b * kMaxE + threadIdx.x] : 0;
    }
    __syncthreads();
    for (int r = threadIdx.x; r < D; r += blockDim.x) {
        float yv[kMaxE];
#pragma unroll
        for (int ki = 0; ki < kMaxE; ki++) yv[ki] = ki < k ? y[(size_t)row_s[ki] * D + r] : 0.f;
        float eo = 0.f;
#pragma unroll
        for (int ki = 0; ki < kMaxE; ki++)
            if (ki < k) eo = __fadd_rn(eo, __fmul_rn(w_s[ki], yv[ki]));
        x[(size_t)b * D + r] = __fadd_rn(x[(size_t)b * D + r], eo);
    }
}

// ------------------------------------------------------------------------------------
// Next token per sequence (one CTA, 1024 threads): the prompt's next id while it lasts
// (sequential prefill, janusdoe.c:3660), else greedy first-index argmax (janusdoe.c:3637,
// 3374-3375) or sample() with temperature and top-k (janusdoe.c:3638-3645) using the
// sequence's own xorshift state.  Advances tok/pos and appends generated ids to history.
struct PickArgs {
    const float *logits;
    int V, ldl;
    float temp;
    int top_k;
    int *tok, *pos;
    uint64_t *rng;
    const int *plen, *prompt;
    int Pmax;
    int *hist, *hist_n;
    int Hmax;
    int *next_out;
    unsigned long long *stats;
    int count_experts;  // batch 1 without route: the election count is the expert count
};
__device__ __forceinline__ uint32_t f2key(float f) {
    uint32_t u = __float_as_uint(f);
    if (u == 0x80000000u) u = 0;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
    return __uint_as_float(u);
}
constexpr int kCandCap = 2048;
static __global__ __launch_bounds__(1024) void k_pick(PickArgs a) {
    const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float *lg = a.logits + (size_t)b * a.ldl;
    const int V = a.V;
    const int p = a.pos[b];
    __shared__ int s_next;
    __shared__ float rv[32];
    __shared__ int ri[32];
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_prefix, s_mask, s_rank;
    __shared__ int cand[kCandCap];
    __shared__ int s_ncand;
    __shared__ int wcount[32];
    const bool from_prompt = a.plen && (p + 1 < a.plen[b]);
    if (from_prompt) {
        if (tid == 0) s_next = a.prompt[(size_t)b * a.Pmax + p + 1];
    } else if (a.temp <= 0.f) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int i = tid; i < V; i += blockDim.x) {
            float v = lg[i];
            if (v > bv || (v == bv && i < bi)) {
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
            float best = rv[0];
            int bidx = ri[0];
            for (int w = 1; w < (int)(blockDim.x >> 5); w++)
                if (rv[w] > best || (rv[w] == best && ri[w] < bidx)) {
                    best = rv[w];
                    bidx = ri[w];
                }
            s_next = bidx == 0x7fffffff ? 0 : bidx;
        }
    } else {
        // logits[i] /= temp, then the top_k-th largest value th by radix select
        const float temp = a.temp;
        const bool use_topk = a.top_k > 0 && a.top_k < V;
        float th = -INFINITY;
        if (use_topk) {
            if (tid == 0) {
                s_prefix = 0;
                s_mask = 0;
                s_rank = (uint32_t)a.top_k;
            }
            for (int shift = 24; shift >= 0; shift -= 8) {
                for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
                __syncthreads();
                uint32_t prefix = s_prefix, mask = s_mask;
                for (int i = tid; i < V; i += blockDim.x) {
                    uint32_t k = f2key(lg[i] / temp);
                    if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1u);
                }
                __syncthreads();
                if (tid == 0) {
                    uint32_t rank = s_rank;
                    for (int d = 255; d >= 0; d--) {
                        if (rank <= hist[d]) {
                            s_prefix = prefix | ((uint32_t)d << shift);
                            s_mask = mask | (255u << shift);
                            break;
                        }
                        rank -= hist[d];
                    }
                    s_rank = rank;
                }
                __syncthreads();
            }
            th = key2f(s_prefix);
        }
        // candidates: !(l < th), compacted in index order
        if (tid == 0) s_ncand = 0;
        __syncthreads();
        bool overflow = false;
        for (int base = 0; base < V; base += blockDim.x) {
            int i = base + tid;
            bool is_c = false;
            if (i < V) {
                float l = lg[i] / temp;
                is_c = !use_topk || !(l < th);
            }
            unsigned m = __ballot_sync(JDG_FULL, is_c);
            if (lane == 0) wcount[warp] = __popc(m);
            __syncthreads();
            int off = s_ncand;
            for (int w = 0; w < warp; w++) off += wcount[w];
            if (is_c) {
                int j = off + __popc(m & ((1u << lane) - 1));
                if (j < kCandCap) cand[j] = i;
            }
            __syncthreads();
            if (tid == 0) {
                int tot = 0;
                for (int w = 0; w < (int)(blockDim.x >> 5); w++) tot += wcount[w];
                s_ncand += tot;
            }
            __syncthreads();
        }
        overflow = s_ncand > kCandCap;
        if (tid == 0) {
            // softmax_n over the masked logits (janusdoe.c:534) restricted to the non-zero
            // terms, summed in index order, then the CDF scan with r = rand_uniform()
            int n = s_ncand;
            float mx = -INFINITY;
            if (!overflow) {
                for (int j = 0; j < n; j++) mx = fmaxf(mx, lg[cand[j]] / temp);
            } else {
                for (int i = 0; i < V; i++) {
                    float l = lg[i] / temp;
                    if (!use_topk || !(l < th)) mx = fmaxf(mx, l);
                }
            }
            float s = 0.f;
            if (!overflow) {
                for (int j = 0; j < n; j++) s = __fadd_rn(s, expf(__fsub_rn(lg[cand[j]] / temp, mx)));
            } else {
                for (int i = 0; i < V; i++) {
                    float l = lg[i] / temp;
                    if (!use_topk || !(l < th)) s = __fadd_rn(s, expf(__fsub_rn(l, mx)));
                }
            }
            uint64_t st = a.rng[b];
            float r = xs_uniform(st);
            a.rng[b] = st;
            int pick = V - 1;
            float cum = 0.f;
            if (r <= 0.f) pick = 0;
            else if (!overflow) {
                for (int j = 0; j < n; j++) {
                    cum = __fadd_rn(cum, expf(__fsub_rn(lg[cand[j]] / temp, mx)) / s);
                    if (cum >= r) {
                        pick = cand[j];
                        break;
                    }
                }
            } else {
                for (int i = 0; i < V; i++) {
                    float l = lg[i] / temp;
                    if (use_topk && l < th) continue;
                    cum = __fadd_rn(cum, expf(__fsub_rn(l, mx)) / s);
                    if (cum >= r) {
                        pick = i;
                        break;
                    }
                }
            }
            s_next = pick;
        }
    }
    __syncthreads();
    if (tid == 0) {
        if (a.stats) {
            atomicAdd(a.stats + 1, (unsigned long long)(p + 1));
            if (b == 0) atomicAdd(a.stats + 2, 1ull);
        }
        int nx = s_next;
        a.tok[b] = nx;
        a.pos[b] = p + 1;
        if (a.next_out) a.next_out[b] = nx;
        if (!from_prompt && a.hist) {
            int hn = a.hist_n[b];
            if (hn < a.Hmax) a.hist[(size_t)b * a.Hmax + hn] = nx;
            a.hist_n[b] = hn + 1;
        }
    }
}

// Tensor-parallel greedy pick: each rank contributed (max, first global index) of its vocab
// slice; the first-index maximum over ranks is the global first-index maximum
// (janusdoe.c:3374-3375).  Prompt and history handling as in k_pick.  One thread per sequence.
static __global__ void k_pick_tp(const float *__restrict__ v, const int *__restrict__ ix, int world, int B, int *tok, int *pos,
                          const int *plen, const int *prompt, int Pmax, int *hist, int *hist_n, int Hmax, int *next_out,
                          unsigned long long *stats) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int r = 0; r < world; r++) {
        float vv = v[r * B + b];
        int ii = ix[r * B + b];
        if (vv > bv || (vv == bv && ii < bi)) {
            bv = vv;
            bi = ii;
        }
    }
    const int p = pos[b];
    if (stats) {
        atomicAdd(stats + 1, (unsigned long long)(p + 1));
        if (b == 0) atomicAdd(stats + 2, 1ull);
    }
    const bool from_prompt = plen && p + 1 < plen[b];
    const int nx = from_prompt ? prompt[(size_t)b * Pmax + p + 1] : (bi == 0x7fffffff ? 0 : bi);
    tok[b] = nx;
    pos[b] = p + 1;
    if (next_out) next_out[b] = nx;
    if (!from_prompt && hist) {
        int hn = hist_n[b];
        if (hn < Hmax) hist[(size_t)b * Hmax + hn] = nx;
        hist_n[b] = hn + 1;
    }
}

}  // namespace jdg

// jdg_b1.cuh — batch-1 decode step as a chain of Programmatic-Dependent-Launch kernels.
//
// Per layer:  QKV (RMSNorm prologue) -> ATTN (RoPE, KV append, split-K partials, last-CTA
// combine) -> WO (+residual, last-CTA parliament election) -> FFN1 (gate/up of the elected
// experts) -> FFN2 (down of the elected experts, last-CTA ordered combine + residual);
// then LMHEAD (final RMSNorm prologue, last-CTA greedy pick).
//
// Every kernel loads the weights it will use into registers BEFORE griddepcontrol.wait, so
// the HBM traffic of kernel N+1 overlaps kernel N; only data written by the immediately
// preceding kernel is read after the wait.  Data written two or more kernels earlier
// (positions, KV history, the election read by FFN2) is complete when a kernel starts,
// because its predecessor triggers its dependents only after its own wait returned.
// The "last CTA" tails use a fence + atomic ticket (no spinning): the CTA that draws the
// final ticket sees every other CTA's writes and finishes the reduction.
#pragma once
#include "jdg_kernels.cuh"

namespace jdg {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void prefetch_l2(const void *p) { asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(p)); }

constexpr int kB1Chunk = 32;  // attention positions per CTA in the batch-1 path

struct B1Args {
    // model
    const float *tok_emb;
    int V, D, H, KVH, HD, hidden, qd, kd, qkvd, max_seq, L, kmax;
    float eps, scale, clamp, inv_clamp;
    int rope_norm;
    const float *rope_cos, *rope_sin;
    // per-layer pointers for this launch
    const float *attn_norm, *ffn_norm, *wqkv, *wo, *w_vote, *w_vote_next;
    const int *alive;
    float temperature;
    const float *const *gu_tab;
    const float *const *dn_tab;
    const float *output, *output_norm;
    int l;
    // state / activations
    const int *tok;
    int *pos;
    float *x, *xb, *qkv, *att, *part, *hbuf, *ybuf, *logits;
    float *kc, *vc;  // layer base
    long kv_bstride;
    int *kcnt, *sel;
    float *selw, *consensus;
    int *tr_k, *tr_sel;
    float *tr_w, *tr_ema;
    unsigned *tickets;     // 1024 counters: [0,32) attention, 32 WO, 48 LM head, 64+ FFN2 row blocks
    float *amax_v;
    int *amax_i;
    float *vpart;          // WO: per-CTA partial votes [gridDim][17] (16 experts + sum of squares)
    float *ffn_inv;        // WO tail: 1/sqrt(mean(x^2)+eps) of the FFN RMSNorm
    unsigned long long *stats;
    int *tok_out, *plen, *prompt, *hist, *hist_n, *next_out;
    int Pmax, Hmax, greedy_pick;
    int *err;
    int embed;             // layer 0: the QKV prologue gathers tok_emb[tok]
};

// ---- warp-parallel parliament election (janusdoe.c:779-838), lane e holds expert e ----
// votes_s[e] holds the fp32 vote of every alive expert; called by every thread of a CTA.
__device__ void b1_election(const B1Args &a, const float *xs, float *votes_s, int warp, int lane, int nwarps) {
    (void)xs;
    (void)nwarps;
    __syncthreads();
    if (warp != 0) return;
    const bool al = lane < kMaxE && a.alive[lane];
    const unsigned am = __ballot_sync(JDG_FULL, al);
    const int na = __popc(am);
    float v = al ? votes_s[lane] : -INFINITY;  // dot + 0.1f * 0 (harmonic state is zero)
    float *cons = a.consensus + a.l;
    int k = 0;
    int my_sel = -1;
    float my_w = 0.f;
    float ema = *cons;
    if (na >= 2) {
        // mean and variance in the reference's sequential order (alive slots ascending)
        float mean = 0.f, var = 0.f;
        for (int e = 0; e < kMaxE; e++) {
            float ve = __shfl_sync(JDG_FULL, v, e);
            if (am & (1u << e)) mean = __fadd_rn(mean, ve);
        }
        mean = mean / (float)na;
        for (int e = 0; e < kMaxE; e++) {
            float ve = __shfl_sync(JDG_FULL, v, e);
            if (am & (1u << e)) {
                float dd = __fsub_rn(ve, mean);
                var = __fadd_rn(var, __fmul_rn(dd, dd));
            }
        }
        var = var / (float)na;
        float cs = fminf(1.0f, sqrtf(__fadd_rn(var, 1e-8f)) / __fadd_rn(fabsf(mean), 1.0f));
        ema = __fadd_rn(__fmul_rn(0.9f, ema), __fmul_rn(0.1f, cs));
        k = (int)__fmul_rn((float)na, __fsub_rn(1.0f, ema));
        if (k < 2) k = 2;
        if (k > na) k = na;
        // top-k by repeated argmax, strict '>' so the lowest slot wins ties (default slot 0)
        bool used = false;
        float wk = 0.f;
        for (int ki = 0; ki < k; ki++) {
            float bv = (al && !used && v > -1e30f) ? v : -1e30f;
            int bi = (al && !used && v > -1e30f) ? lane : 0x7fffffff;
            for (int o = 16; o; o >>= 1) {
                float ov = __shfl_xor_sync(JDG_FULL, bv, o);
                int oi = __shfl_xor_sync(JDG_FULL, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (bi == 0x7fffffff) bi = 0;
            if (lane == bi) used = true;
            float wsel = __shfl_sync(JDG_FULL, v, bi);
            if (lane == ki) {
                my_sel = bi;
                wk = wsel;
            }
        }
        float temp = a.temperature > 0.05f ? a.temperature : 1.0f;
        float mx = -INFINITY;
        for (int i = 0; i < k; i++) mx = fmaxf(mx, __shfl_sync(JDG_FULL, wk, i));
        float ex = lane < k ? expf(__fsub_rn(wk, mx) / temp) : 0.f;
        float sum = 0.f;
        for (int i = 0; i < k; i++) sum = __fadd_rn(sum, __shfl_sync(JDG_FULL, ex, i));
        my_w = lane < k ? ex / sum : 0.f;
        if (lane == 0) *cons = ema;
    }
    if (lane < kMaxE) {
        a.sel[lane] = lane < k ? my_sel : -1;
        a.selw[lane] = lane < k ? my_w : 0.f;
        a.tr_sel[(size_t)a.l * kMaxE + lane] = lane < k ? my_sel : -1;
        a.tr_w[(size_t)a.l * kMaxE + lane] = lane < k ? my_w : 0.f;
    }
    if (lane == 0) {
        a.kcnt[0] = k;
        a.tr_k[a.l] = k;
        a.tr_ema[a.l] = ema;
        atomicAdd(a.stats, (unsigned long long)k);
    }
}

// fence + ticket: returns true in the one CTA that arrives last (all threads of it)
__device__ __forceinline__ bool last_cta(unsigned *ctr, unsigned expected) {
    __shared__ unsigned s_ticket;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_ticket = atomicAdd(ctr, 1u);
    __syncthreads();
    bool last = s_ticket == expected - 1;
    if (last) __threadfence();
    return last;
}

// ---------------------------------------------------------------------------------
// QKV: qkv = Wqkv . rmsnorm(x, attn_norm); layer 0 first gathers x = tok_emb[tok].
// 4 warps x 1 row; NV = D/128 float4 per lane held in registers.
template <int NV>
__global__ __launch_bounds__(128) void k_b1_qkv(B1Args a) {
    __shared__ __align__(16) float xs[NV * 128];
    __shared__ float red[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row = blockIdx.x * 4 + warp;
    float4 w[NV];
    if (row < a.qkvd) {
        const float *wr = a.wqkv + (size_t)row * a.D;
#pragma unroll
        for (int j = 0; j < NV; j++) w[j] = ld_stream4(wr + 4 * (lane + 32 * j));
    }
    if (blockIdx.x == 0) {  // warm L2 with this layer's vote rows for the WO tail
        for (int i = threadIdx.x; i < kMaxE * a.D / 32; i += blockDim.x) prefetch_l2(a.w_vote + (size_t)i * 32);
    }
    pdl_wait();
    pdl_trigger();
    const float *src = a.x;
    if (a.embed) {
        int t = a.tok[0];
        if (t < 0 || t >= a.V) {
            if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(a.err, JDG_ERR_TOKEN);
            t = 0;
        }
        src = a.tok_emb + (size_t)t * a.D;
    }
    float ss = 0.f;
    for (int i = threadIdx.x; i < a.D / 4; i += blockDim.x) {
        float4 v = reinterpret_cast<const float4 *>(src)[i];
        reinterpret_cast<float4 *>(xs)[i] = v;
        ss = dot4(v, v, ss);
        if (a.embed && blockIdx.x == 0) reinterpret_cast<float4 *>(a.x)[i] = v;
    }
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)a.D + a.eps);
    if (row >= a.qkvd) return;
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < NV; j++) {
        int i4 = lane + 32 * j;
        float4 xv = reinterpret_cast<const float4 *>(xs)[i4];
        float4 nw = reinterpret_cast<const float4 *>(a.attn_norm)[i4];
        xv.x = __fmul_rn(__fmul_rn(xv.x, inv), nw.x);
        xv.y = __fmul_rn(__fmul_rn(xv.y, inv), nw.y);
        xv.z = __fmul_rn(__fmul_rn(xv.z, inv), nw.z);
        xv.w = __fmul_rn(__fmul_rn(xv.w, inv), nw.w);
        acc = dot4(w[j], xv, acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) a.qkv[row] = acc;
}

// ---------------------------------------------------------------------------------
// ATTN: grid (ceil(max_seq/32), KVH).  CTA (c, g) owns positions [32c, 32c+32) of KV head
// g.  History rows (t < pos) are loaded before the wait; the row at pos is RoPE'd from
// qkv, appended to the cache, and used directly.  Partials (o, m, l) per head; the last
// CTA of head group g merges them into att.  Scores: s = (q.k)*scale, clamp*tanh(s/clamp).
template <int HD>
__global__ __launch_bounds__(128) void k_b1_attn(B1Args a) {
    constexpr int RS = HD + 4;  // padded row stride (conflict-free float4 reads)
    __shared__ __align__(16) float ks[kB1Chunk][RS];
    __shared__ __align__(16) float vs[kB1Chunk][RS];
    __shared__ __align__(16) float qs[kMaxHG][HD];
    __shared__ float ps[kMaxHG][kB1Chunk];
    const int c = blockIdx.x, g = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int p = a.pos[0];
    const int t0 = c * kB1Chunk;
    const int hg = a.H / a.KVH, kd = a.kd;
    const int nc_total = p / kB1Chunk + 1;
    if (t0 > p) {
        pdl_wait();
        pdl_trigger();
        return;
    }
    const int nt = min(kB1Chunk, p + 1 - t0);
    // history rows t0..min(t0+32, p)-1 straight into shared memory (before the wait)
    const float *kb = a.kc + (size_t)t0 * kd + (size_t)g * HD;
    const float *vb = a.vc + (size_t)t0 * kd + (size_t)g * HD;
    const int nh = min(nt, p - t0);  // rows already in the cache
    for (int i = tid; i < nh * (HD / 4); i += blockDim.x) {
        int t = i / (HD / 4), d4 = i % (HD / 4);
        *reinterpret_cast<float4 *>(&ks[t][4 * d4]) = __ldcg(reinterpret_cast<const float4 *>(kb + (size_t)t * kd) + d4);
        *reinterpret_cast<float4 *>(&vs[t][4 * d4]) = __ldcg(reinterpret_cast<const float4 *>(vb + (size_t)t * kd) + d4);
    }
    pdl_wait();
    pdl_trigger();
    if (p < 0 || p >= a.max_seq) {
        if (tid == 0 && c == 0 && g == 0) atomicOr(a.err, JDG_ERR_POS);
        return;
    }
    const int half = HD / 2;
    const float *ct = a.rope_cos + (size_t)p * half, *st = a.rope_sin + (size_t)p * half;
    // RoPE the q heads of this group (and k at p if this chunk holds p)
    const bool has_p = (p - t0) < kB1Chunk;
    const int nrot = (hg + (has_p ? 1 : 0)) * half;
    for (int idx = tid; idx < nrot; idx += blockDim.x) {
        int j = idx / half, i = idx % half;
        int i0 = a.rope_norm ? 2 * i : i, i1 = a.rope_norm ? 2 * i + 1 : i + half;
        const float *src = j < hg ? a.qkv + (size_t)(g * hg + j) * HD : a.qkv + a.qd + (size_t)g * HD;
        float x0 = src[i0], x1 = src[i1], cc = ct[i], sn = st[i];
        float y0 = __fsub_rn(__fmul_rn(x0, cc), __fmul_rn(x1, sn));
        float y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cc));
        if (j < hg) {
            qs[j][i0] = y0;
            qs[j][i1] = y1;
        } else {
            ks[p - t0][i0] = y0;
            ks[p - t0][i1] = y1;
        }
    }
    if (has_p) {
        const float *vsrc = a.qkv + a.qd + kd + (size_t)g * HD;
        for (int d = tid; d < HD; d += blockDim.x) vs[p - t0][d] = vsrc[d];
    }
    __syncthreads();
    if (has_p) {  // append k (roped) and v at p
        float *kdst = a.kc + (size_t)p * kd + (size_t)g * HD, *vdst = a.vc + (size_t)p * kd + (size_t)g * HD;
        for (int d = tid; d < HD; d += blockDim.x) {
            kdst[d] = ks[p - t0][d];
            vdst[d] = vs[p - t0][d];
        }
    }
    // scores: warp w handles heads w, w+4; lane = position
    for (int j = warp; j < hg; j += 4) {
        float s = -INFINITY;
        if (lane < nt) {
            float d = 0.f;
#pragma unroll
            for (int d4 = 0; d4 < HD / 4; d4++)
                d = dot4(*reinterpret_cast<const float4 *>(&qs[j][4 * d4]), *reinterpret_cast<const float4 *>(&ks[lane][4 * d4]), d);
            s = __fmul_rn(d, a.scale);
            if (a.clamp > 0.f) s = __fmul_rn(a.clamp, tanhf(__fmul_rn(s, a.inv_clamp)));
        }
        float m = warp_max(s);
        float e = lane < nt ? expf(s - m) : 0.f;
        float l = warp_sum(e);
        ps[j][lane] = e;
        __syncwarp();
        // o[d] for this head: lane owns HD/32 dims
        constexpr int E = HD / 32;
        float o[E];
#pragma unroll
        for (int q = 0; q < E; q++) o[q] = 0.f;
        for (int t = 0; t < nt; t++) {
            float pt = ps[j][t];
#pragma unroll
            for (int q = 0; q < E; q++) o[q] = fmaf(pt, vs[t][lane * E + q], o[q]);
        }
        float *dst = a.part + ((size_t)(g * hg + j) * (a.max_seq / kB1Chunk + 1) + c) * (HD + 2);
#pragma unroll
        for (int q = 0; q < E; q++) dst[lane * E + q] = o[q];
        if (lane == 0) {
            dst[HD] = m;
            dst[HD + 1] = l;
        }
    }
    // last CTA of this KV head merges the chunks of its query heads:
    // f_c = e^{m_c - M} / sum_c l_c e^{m_c - M};  att = sum_c o_c f_c
    if (!last_cta(a.tickets + g, nc_total)) return;
    const int ncs = a.max_seq / kB1Chunk + 1;
    __shared__ float fm[kMaxHG][kB1Chunk + 2];
    for (int idx = tid; idx < hg * nc_total; idx += blockDim.x) {
        int j = idx / nc_total, cc = idx % nc_total;
        fm[j][cc] = __ldcg(a.part + ((size_t)(g * hg + j) * ncs + cc) * (HD + 2) + HD);
        ps[j][cc] = __ldcg(a.part + ((size_t)(g * hg + j) * ncs + cc) * (HD + 2) + HD + 1);
    }
    __syncthreads();
    for (int j = warp; j < hg; j += 4) {
        float m = lane < nc_total ? fm[j][lane] : -INFINITY;
        float M = warp_max(m);
        float f = lane < nc_total ? expf(m - M) : 0.f;
        float S = warp_sum(lane < nc_total ? ps[j][lane] * f : 0.f);
        if (lane < nc_total) fm[j][lane] = f / S;
    }
    __syncthreads();
    for (int idx = tid; idx < hg * HD; idx += blockDim.x) {
        int j = idx / HD, d = idx % HD, h = g * hg + j;
        const float *pp = a.part + (size_t)h * ncs * (HD + 2) + d;
        float o = 0.f;
#pragma unroll 8
        for (int cc = 0; cc < nc_total; cc++) o = fmaf(__ldcg(pp + cc * (HD + 2)), fm[j][cc], o);
        a.att[h * HD + d] = o;
    }
    if (tid == 0) a.tickets[g] = 0;
}

// ---------------------------------------------------------------------------------
// WO: x += Wo . att (janusdoe.c:911-912).  Each CTA also emits, for its 4 rows r, the
// partial sums  sum_r x_r^2  and  sum_r (w_vote[e][r] * ffn_norm[r]) * x_r  for the 16
// vote rows; the last CTA reduces them (vote_e = inv * sum, the factored form of
// w_vote[e] . rmsnorm(x, ffn_norm), janusdoe.c:915, 795-797) and runs the election.
template <int NV>
__global__ __launch_bounds__(128) void k_b1_wo(B1Args a) {
    __shared__ __align__(16) float xs[NV * 128];
    __shared__ float xnew[4];
    __shared__ float votes_s[kMaxE];
    __shared__ float red[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row = blockIdx.x * 4 + warp;
    float4 w[NV];
    if (row < a.D) {
        const float *wr = a.wo + (size_t)row * a.qd;
#pragma unroll
        for (int j = 0; j < NV; j++) w[j] = ld_stream4(wr + 4 * (lane + 32 * j));
    }
    // vote-row coefficients for this CTA's rows: thread t < 64 -> (expert t/4, row t%4)
    float wv = 0.f;
    if (threadIdx.x < 64) {
        int e = threadIdx.x >> 2, r = blockIdx.x * 4 + (threadIdx.x & 3);
        if (r < a.D && a.alive[e]) wv = __fmul_rn(a.w_vote[(size_t)e * a.D + r], a.ffn_norm[r]);
    }
    pdl_wait();
    pdl_trigger();
    for (int i = threadIdx.x; i < a.qd / 4; i += blockDim.x)
        reinterpret_cast<float4 *>(xs)[i] = __ldcg(reinterpret_cast<const float4 *>(a.att) + i);
    __syncthreads();
    float xn = 0.f;
    if (row < a.D) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < NV; j++) acc = dot4(w[j], reinterpret_cast<const float4 *>(xs)[lane + 32 * j], acc);
        acc = warp_sum(acc);
        xn = __fadd_rn(a.x[row], acc);
        if (lane == 0) a.x[row] = xn;
    }
    if (lane == 0) xnew[warp] = xn;
    __syncthreads();
    if (threadIdx.x < 64) {
        float pv = wv * xnew[threadIdx.x & 3];
        pv += __shfl_xor_sync(0xffffffffu, pv, 1);
        pv += __shfl_xor_sync(0xffffffffu, pv, 2);
        if ((threadIdx.x & 3) == 0) a.vpart[(size_t)blockIdx.x * 17 + (threadIdx.x >> 2)] = pv;
    }
    if (threadIdx.x == 64) {
        float ss = 0.f;
        for (int q = 0; q < 4; q++) ss = fmaf(xnew[q], xnew[q], ss);
        a.vpart[(size_t)blockIdx.x * 17 + 16] = ss;
    }
    if (!last_cta(a.tickets + 32, gridDim.x)) return;
    // reduce partials: warp w sums quantities w, w+4, ... (17 of them) over the CTAs
    const int nb = gridDim.x;
    __shared__ float tot[17];
    for (int qn = warp; qn < 17; qn += 4) {
        float v = 0.f;
        for (int b = lane; b < nb; b += 32) v += __ldcg(a.vpart + (size_t)b * 17 + qn);
        v = warp_sum(v);
        if (lane == 0) tot[qn] = v;
    }
    __syncthreads();
    const float inv = 1.0f / sqrtf(tot[16] / (float)a.D + a.eps);
    if (threadIdx.x < kMaxE) votes_s[threadIdx.x] = __fmul_rn(inv, tot[threadIdx.x]);
    if (threadIdx.x == 0) *a.ffn_inv = inv;
    __syncthreads();
    b1_election(a, nullptr, votes_s, warp, lane, 4);
    if (threadIdx.x == 0) a.tickets[32] = 0;
    (void)red;
}

// ---------------------------------------------------------------------------------
// FFN1: h_ki[i] = silu(Wg_e[i].xb) * (Wu_e[i].xb) for elected experts (janusdoe.c:923-925).
// grid (ceil(hidden/4), kmax); rows (2i, 2i+1) of the interleaved gate/up matrix.
template <int NV>
__global__ __launch_bounds__(128) void k_b1_ffn1(B1Args a) {
    __shared__ __align__(16) float xs[NV * 128];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ki = blockIdx.y;
    const int i = blockIdx.x * 4 + warp;
    pdl_wait();
    pdl_trigger();
    const int k = __ldcg(a.kcnt);
    if (ki >= k) return;
    const int e = __ldcg(a.sel + ki);
    const float *W = (e >= 0 && e < kMaxE) ? a.gu_tab[e] : nullptr;
    if (W == nullptr) {
        if (threadIdx.x == 0) atomicOr(a.err, JDG_ERR_ROUTE);
        return;
    }
    float4 wg[NV], wu[NV];
    if (i < a.hidden) {
        const float *g = W + (size_t)(2 * i) * a.D, *u = g + a.D;
#pragma unroll
        for (int j = 0; j < NV; j++) {
            wg[j] = ld_stream4(g + 4 * (lane + 32 * j));
            wu[j] = ld_stream4(u + 4 * (lane + 32 * j));
        }
    }
    {
        const float inv = __ldcg(a.ffn_inv);
        for (int q = threadIdx.x; q < a.D; q += blockDim.x) {
            float v = __fmul_rn(__fmul_rn(__ldcg(a.x + q), inv), a.ffn_norm[q]);
            xs[q] = v;
            if (blockIdx.x == 0 && blockIdx.y == 0) a.xb[q] = v;
        }
    }
    __syncthreads();
    if (i >= a.hidden) return;
    float ag = 0.f, au = 0.f;
#pragma unroll
    for (int j = 0; j < NV; j++) {
        float4 xv = reinterpret_cast<const float4 *>(xs)[lane + 32 * j];
        ag = dot4(wg[j], xv, ag);
        au = dot4(wu[j], xv, au);
    }
    ag = warp_sum(ag);
    au = warp_sum(au);
    if (lane == 0) a.hbuf[(size_t)ki * a.hidden + i] = __fmul_rn(silu_ref(ag), au);
}

// ---------------------------------------------------------------------------------
// FFN2: y_ki[r] = Wd_e[r] . h_ki; the last CTA of each 4-row block adds
// sum_ki w_ki * y_ki[r] in election order to x (janusdoe.c:926-929).
// grid (D/4, kmax).  The election (written by WO, two kernels earlier) is read before the
// wait so the down rows stream while FFN1 is still running.
template <int NH>
__global__ __launch_bounds__(128) void k_b1_ffn2(B1Args a) {
    __shared__ __align__(16) float hs[NH * 128];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ki = blockIdx.y, rb = blockIdx.x;
    const int r = rb * 4 + warp;
    const int k = __ldcg(a.kcnt);
    float4 w[NH];
    const int e = ki < k ? __ldcg(a.sel + ki) : -1;
    const float *W = (e >= 0 && e < kMaxE) ? a.dn_tab[e] : nullptr;
    if (W && r < a.D) {
        const float *wr = W + (size_t)r * a.hidden;
#pragma unroll
        for (int j = 0; j < NH; j++) w[j] = ld_stream4(wr + 4 * (lane + 32 * j));
    }
    pdl_wait();
    pdl_trigger();
    if (ki >= k) return;
    if (W == nullptr && threadIdx.x == 0) atomicOr(a.err, JDG_ERR_ROUTE);
    for (int q = threadIdx.x; q < a.hidden / 4; q += blockDim.x)
        reinterpret_cast<float4 *>(hs)[q] = __ldcg(reinterpret_cast<const float4 *>(a.hbuf + (size_t)ki * a.hidden) + q);
    __syncthreads();
    if (r < a.D) {
        float acc = 0.f;
        if (W) {
#pragma unroll
            for (int j = 0; j < NH; j++) acc = dot4(w[j], reinterpret_cast<const float4 *>(hs)[lane + 32 * j], acc);
            acc = warp_sum(acc);
        }
        if (lane == 0) a.ybuf[(size_t)ki * a.D + r] = acc;
    }
    if (!last_cta(a.tickets + 64 + rb, k)) return;
    if (threadIdx.x < 4) {
        int rr = rb * 4 + threadIdx.x;
        if (rr < a.D) {
            float eo = 0.f;
            for (int q = 0; q < k; q++) eo = __fadd_rn(eo, __fmul_rn(__ldcg(a.selw + q), __ldcg(a.ybuf + (size_t)q * a.D + rr)));
            a.x[rr] = __fadd_rn(a.x[rr], eo);
        }
    }
    if (threadIdx.x == 0) a.tickets[64 + rb] = 0;
}

// ---------------------------------------------------------------------------------
// LMHEAD: logits = Wout . rmsnorm(x, output_norm) (janusdoe.c:931-932).  Per-CTA argmax
// partials; with greedy_pick the last CTA takes the first-index maximum (janusdoe.c:3637)
// or the prompt's next id, and advances tok/pos/history.
template <int NV>
__global__ __launch_bounds__(128) void k_b1_lmhead(B1Args a) {
    __shared__ __align__(16) float xs[NV * 128];
    __shared__ float red[32];
    __shared__ float bv_s[4];
    __shared__ int bi_s[4];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row0 = blockIdx.x * 8 + warp * 2;  // two rows per warp
    float4 w[2][NV];
#pragma unroll
    for (int r = 0; r < 2; r++)
        if (row0 + r < a.V) {
            const float *wr = a.output + (size_t)(row0 + r) * a.D;
#pragma unroll
            for (int j = 0; j < NV; j++) w[r][j] = ld_stream4(wr + 4 * (lane + 32 * j));
        }
    pdl_wait();
    pdl_trigger();
    float ss = 0.f;
    for (int i = threadIdx.x; i < a.D / 4; i += blockDim.x) {
        float4 v = __ldcg(reinterpret_cast<const float4 *>(a.x) + i);
        reinterpret_cast<float4 *>(xs)[i] = v;
        ss = dot4(v, v, ss);
    }
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)a.D + a.eps);
    float acc[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < NV; j++) {
        int i4 = lane + 32 * j;
        float4 xv = reinterpret_cast<const float4 *>(xs)[i4];
        float4 nw = reinterpret_cast<const float4 *>(a.output_norm)[i4];
        xv.x = __fmul_rn(__fmul_rn(xv.x, inv), nw.x);
        xv.y = __fmul_rn(__fmul_rn(xv.y, inv), nw.y);
        xv.z = __fmul_rn(__fmul_rn(xv.z, inv), nw.z);
        xv.w = __fmul_rn(__fmul_rn(xv.w, inv), nw.w);
#pragma unroll
        for (int r = 0; r < 2; r++) acc[r] = dot4(w[r][j], xv, acc[r]);
    }
    float val = -INFINITY;
    int vi = 0x7fffffff;
#pragma unroll
    for (int r = 0; r < 2; r++) {
        float v = warp_sum(acc[r]);
        if (row0 + r < a.V) {
            if (lane == 0) a.logits[row0 + r] = v;
            if (v > val) {
                val = v;
                vi = row0 + r;
            }
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
        for (int q = 1; q < 4; q++)
            if (bv_s[q] > bv) {
                bv = bv_s[q];
                bi = bi_s[q];
            }
        a.amax_v[blockIdx.x] = bv;
        a.amax_i[blockIdx.x] = bi;
    }
    if (!a.greedy_pick) return;
    if (!last_cta(a.tickets + 48, gridDim.x)) return;
    // first-index maximum over CTA partials (CTAs cover increasing rows)
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int q = threadIdx.x; q < (int)gridDim.x; q += blockDim.x) {
        float v = __ldcg(a.amax_v + q);
        int ix = __ldcg(a.amax_i + q);
        if (v > bv || (v == bv && ix < bi)) {
            bv = v;
            bi = ix;
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
        int p = a.pos[0];
        atomicAdd(a.stats + 1, (unsigned long long)(p + 1));
        atomicAdd(a.stats + 2, 1ull);
        bool from_prompt = a.plen && p + 1 < a.plen[0];
        int nx = from_prompt ? a.prompt[p + 1] : (bi_s[0] == 0x7fffffff ? 0 : bi_s[0]);
        a.tok_out[0] = nx;
        a.pos[0] = p + 1;
        if (a.next_out) a.next_out[0] = nx;
        if (!from_prompt && a.hist) {
            int hn = a.hist_n[0];
            if (hn < a.Hmax) a.hist[hn] = nx;
            a.hist_n[0] = hn + 1;
        }
        a.tickets[48] = 0;
    }
}

}  // namespace jdg

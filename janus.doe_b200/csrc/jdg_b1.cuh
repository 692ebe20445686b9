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
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// Optional timeline (engine debug): per kernel slot, earliest CTA entry, earliest return
// from griddepcontrol.wait, latest CTA exit.
struct TlMark {
    unsigned long long *slot;
    __device__ TlMark(unsigned long long *tl, int idx) : slot(tl ? tl + 3 * idx : nullptr) {
        if (slot && threadIdx.x == 0) atomicMin(slot, gtimer());
    }
    __device__ void waited() {
        if (slot && threadIdx.x == 0) atomicMin(slot + 1, gtimer());
    }
    __device__ ~TlMark() {
        if (slot && threadIdx.x == 0) atomicMax(slot + 2, gtimer());
    }
};
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void prefetch_l2(const void *p) { asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(p)); }

constexpr int kB1Chunk = 128;  // attention positions per CTA in the batch-1 path

// Copy n4 float4 (n4 <= 128*MAXPT) from global (L2-coherent loads) to shared memory with
// every load issued before the first store, so the latency is paid once.
template <int MAXPT>
__device__ __forceinline__ void vec_to_smem(float *dst, const float *src, int n4) {
    float4 r[MAXPT];
#pragma unroll
    for (int j = 0; j < MAXPT; j++) {
        int i = threadIdx.x + 128 * j;
        if (i < n4) r[j] = __ldcg(reinterpret_cast<const float4 *>(src) + i);
    }
#pragma unroll
    for (int j = 0; j < MAXPT; j++) {
        int i = threadIdx.x + 128 * j;
        if (i < n4) reinterpret_cast<float4 *>(dst)[i] = r[j];
    }
}
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

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
    float *vpart;          // WO: per-CTA partial votes [nparts][17] (16 experts + sum of squares)
    int nparts;            // WO grid size
    float *ema_new;        // FFN1 CTA 0: this layer's updated EMA, committed by the next kernel
    int combine;           // prologue adds the previous layer's expert outputs to x
    const float *x_prev;   // residual after the previous layer's attention (ping-pong partner of x)
    int n_prev;            // alive experts of the previous layer (expert-output slots to combine)
    float *ffn_inv;        // WO tail: 1/sqrt(mean(x^2)+eps) of the FFN RMSNorm
    unsigned long long *stats;
    const float **sel_gu, **sel_dn;  // weight pointers of the elected experts, in election order
    int *tok_out, *plen, *prompt, *hist, *hist_n, *next_out;
    int Pmax, Hmax, greedy_pick;
    int *err;
    int embed;             // layer 0: the QKV prologue gathers tok_emb[tok]
    unsigned long long *tl;  // optional timeline [kernel][3]
};

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

// ---- parliament election from WO's partial votes (janusdoe.c:779-838) ---------------
// Every CTA that calls this reduces the same partials in the same fixed order, so all of
// them obtain bit-identical elections.  Called by all 128 threads; results in shared.
struct ElectOut {
    int k;
    int sel[kMaxE];
    float w[kMaxE];
    float ema;
    float inv;  // 1/sqrt(mean(x^2)+eps) of the FFN RMSNorm
};
static __device__ void b1_elect(const B1Args &a, ElectOut &eo, const float cons_in) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = a.nparts;  // <= 256
    __shared__ float tot[4][17];
    __shared__ float votes_s[kMaxE];
    __shared__ int alive_s[kMaxE];
    {
        float v0[17], v1[17];
        const int b0 = threadIdx.x, b1 = threadIdx.x + 128;
#pragma unroll
        for (int q = 0; q < 17; q++) {
            v0[q] = b0 < nb ? __ldcg(a.vpart + (size_t)q * nb + b0) : 0.f;
            v1[q] = b1 < nb ? __ldcg(a.vpart + (size_t)q * nb + b1) : 0.f;
        }
        if (threadIdx.x < kMaxE) alive_s[threadIdx.x] = a.alive[threadIdx.x];
#pragma unroll
        for (int q = 0; q < 17; q++) {
            float v = warp_sum(__fadd_rn(v0[q], v1[q]));
            if (lane == 0) tot[warp][q] = v;
        }
    }
    __syncthreads();
    if (threadIdx.x < 17)
        tot[0][threadIdx.x] = __fadd_rn(__fadd_rn(tot[0][threadIdx.x], tot[1][threadIdx.x]),
                                        __fadd_rn(tot[2][threadIdx.x], tot[3][threadIdx.x]));
    __syncthreads();
    if (a.tl && threadIdx.x == 0) atomicMax(a.tl + 3 * (124 + a.l) + 2, gtimer());
    // election on warp 0; every lane evaluates the scalar election on its own registers
    // (votes read once from shared memory), lane 0 publishes.  Loops over the election
    // slots are not unrolled, loops over the 16 expert slots are.
    if (warp == 0) {
        const float inv = 1.0f / sqrtf(tot[0][16] / (float)a.D + a.eps);
        float v[kMaxE];
        unsigned am = 0;
#pragma unroll
        for (int e = 0; e < kMaxE; e++) {
            v[e] = __fmul_rn(inv, tot[0][e]);  // dot + 0.1f * 0 (harmonic state is zero)
            if (alive_s[e]) am |= 1u << e;
        }
        const int na = __popc(am);
        float ema = cons_in;
        int k = 0;
        if (na >= 2) {
            float mean = 0.f, var = 0.f;
#pragma unroll
            for (int e = 0; e < kMaxE; e++)
                if (am & (1u << e)) mean = __fadd_rn(mean, v[e]);
            mean = mean / (float)na;
#pragma unroll
            for (int e = 0; e < kMaxE; e++)
                if (am & (1u << e)) {
                    float dd = __fsub_rn(v[e], mean);
                    var = __fadd_rn(var, __fmul_rn(dd, dd));
                }
            var = var / (float)na;
            float cs = fminf(1.0f, sqrtf(__fadd_rn(var, 1e-8f)) / __fadd_rn(fabsf(mean), 1.0f));
            ema = __fadd_rn(__fmul_rn(0.9f, ema), __fmul_rn(0.1f, cs));
            k = (int)__fmul_rn((float)na, __fsub_rn(1.0f, ema));
            if (k < 2) k = 2;
            if (k > na) k = na;
            unsigned used = 0;
            float mx = -INFINITY;
#pragma unroll 1
            for (int ki = 0; ki < k; ki++) {
                float bv = -1e30f, vb = 0.f;
                int bi = 0;
#pragma unroll
                for (int e = 0; e < kMaxE; e++)
                    if ((am & ~used & (1u << e)) && v[e] > bv) {
                        bv = v[e];
                        bi = e;
                    }
#pragma unroll
                for (int e = 0; e < kMaxE; e++)
                    if (e == bi) vb = v[e];
                used |= 1u << bi;
                mx = fmaxf(mx, vb);
                if (lane == 0) {
                    eo.sel[ki] = bi;
                    eo.w[ki] = vb;
                }
            }
            __syncwarp();
            const float temp = a.temperature > 0.05f ? a.temperature : 1.0f;
            // lanes < k exponentiate their slot; lane 0 sums in election order
            const float ex = lane < k ? expf(__fsub_rn(eo.w[lane], mx) / temp) : 0.f;
            __syncwarp();
            if (lane < k) eo.w[lane] = ex;
            __syncwarp();
            float sum = 0.f;
#pragma unroll 1
            for (int i = 0; i < k; i++) sum = __fadd_rn(sum, eo.w[i]);
            __syncwarp();
            if (lane < k) eo.w[lane] = ex / sum;
        }
        if (lane >= k && lane < kMaxE) {
            eo.sel[lane] = -1;
            eo.w[lane] = 0.f;
        }
        if (lane == 0) {
            eo.k = k;
            eo.ema = ema;
            eo.inv = inv;
        }
    }
    __syncthreads();
}

// x = x_prev + sum_ki w_ki * y_ki in election order (janusdoe.c:927-929), and commit the
// previous layer's EMA (deferred so that no reader of this layer's EMA sees the update).
// Loads the result into xs; CTA 0 stores it to x.  x and x_prev are different buffers
// (layer parity), so no CTA reads what another CTA of the same kernel writes.
template <int NV>
__device__ __forceinline__ void b1_load_x(const B1Args &a, float *xs) {
    const int D4 = a.D / 4;
    float4 xr[(NV + 3) / 4];
#pragma unroll
    for (int j = 0; j < (NV + 3) / 4; j++) {
        int i = threadIdx.x + 128 * j;
        if (i < D4) xr[j] = __ldcg(reinterpret_cast<const float4 *>(a.combine ? a.x_prev : a.x) + i);
    }
    if (a.combine) {
        // expert outputs of the previous layer: slots >= k carry weight 0 (and finite
        // values), so every slot below the layer's alive count is loaded up front
        const int np = a.n_prev;
        float wk[kMaxE];
#pragma unroll
        for (int q = 0; q < kMaxE; q++) wk[q] = q < np ? __ldcg(a.selw + q) : 0.f;
#pragma unroll
        for (int j = 0; j < (NV + 3) / 4; j++) {
            int i = threadIdx.x + 128 * j;
            if (i >= D4) continue;
            float4 eo = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int q0 = 0; q0 < np; q0 += 8) {
                float4 y[8];
#pragma unroll
                for (int q = 0; q < 8; q++)
                    if (q0 + q < np) y[q] = __ldcg(reinterpret_cast<const float4 *>(a.ybuf + (size_t)(q0 + q) * a.D) + i);
#pragma unroll
                for (int q = 0; q < 8; q++)
                    if (q0 + q < np && wk[q0 + q] != 0.f) {
                        const float wq = wk[q0 + q];
                        eo.x = __fadd_rn(eo.x, __fmul_rn(wq, y[q].x));
                        eo.y = __fadd_rn(eo.y, __fmul_rn(wq, y[q].y));
                        eo.z = __fadd_rn(eo.z, __fmul_rn(wq, y[q].z));
                        eo.w = __fadd_rn(eo.w, __fmul_rn(wq, y[q].w));
                    }
            }
            xr[j].x = __fadd_rn(xr[j].x, eo.x);
            xr[j].y = __fadd_rn(xr[j].y, eo.y);
            xr[j].z = __fadd_rn(xr[j].z, eo.z);
            xr[j].w = __fadd_rn(xr[j].w, eo.w);
        }
        if (blockIdx.x == 0 && threadIdx.x == 0) a.consensus[a.l - 1] = __ldcg(a.ema_new);
    }
#pragma unroll
    for (int j = 0; j < (NV + 3) / 4; j++) {
        int i = threadIdx.x + 128 * j;
        if (i < D4) {
            reinterpret_cast<float4 *>(xs)[i] = xr[j];
            if (blockIdx.x == 0 && (a.combine || a.embed)) reinterpret_cast<float4 *>(a.x)[i] = xr[j];
        }
    }
}

// ---------------------------------------------------------------------------------
// QKV: qkv = Wqkv . rmsnorm(x, attn_norm); layer 0 first gathers x = tok_emb[tok], later
// layers first add the previous layer's expert outputs.
template <int NV>
static __global__ __launch_bounds__(128) void k_b1_qkv(B1Args a) {
    TlMark tlm(a.tl, a.l * 5 + 0);
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
    pdl_wait();
    tlm.waited();
    pdl_trigger();
    if (a.embed) {
        int t = a.tok[0];
        if (t < 0 || t >= a.V) {
            if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(a.err, JDG_ERR_TOKEN);
            t = 0;
        }
        B1Args b = a;
        b.x = const_cast<float *>(a.tok_emb + (size_t)t * a.D);
        b.combine = 0;
        b.embed = 0;
        b1_load_x<NV>(b, xs);
        if (blockIdx.x == 0)
            for (int i = threadIdx.x; i < a.D / 4; i += 128)
                reinterpret_cast<float4 *>(a.x)[i] = reinterpret_cast<const float4 *>(xs)[i];
    } else {
        b1_load_x<NV>(a, xs);
    }
    __syncthreads();
    float ss = 0.f;
    for (int i = threadIdx.x; i < a.D / 4; i += blockDim.x) {
        float4 v = reinterpret_cast<const float4 *>(xs)[i];
        ss = dot4(v, v, ss);
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
// ATTN: grid (ceil(max_seq/128), KVH).  CTA (c, g) owns positions [128c, 128c+128) of KV
// head g: history rows (t < pos) are copied to shared memory before the wait; the row at
// pos is RoPE'd from qkv, appended to the cache and used directly.  Writes per-head
// partials (unnormalised o, chunk max m, chunk sum l); WO merges them.
// s = (q.k)*scale, then clamp*tanh(s/clamp) (janusdoe.c:899-910).
// One attention CTA: positions [128c, 128c+128) of KV head g (called by k_b1_attn and by
// the host chain's attention kernel).  Dynamic shared memory: 2*128*(HD+4) floats.
template <int HD>
__device__ __forceinline__ void b1_attn_cta(const B1Args &a, const int c, const int g, TlMark &tlm) {
    constexpr int RS = HD + 4;  // padded row stride (conflict-free float4 reads)
    constexpr int CH = kB1Chunk;
    extern __shared__ __align__(16) float dsm[];
    float(*ks)[RS] = reinterpret_cast<float(*)[RS]>(dsm);
    float(*vs)[RS] = reinterpret_cast<float(*)[RS]>(dsm + CH * RS);
    __shared__ __align__(16) float qs[kMaxHG][HD];
    __shared__ float ps[kMaxHG][CH];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int p = a.pos[0];
    const int t0 = c * CH;
    const int hg = a.H / a.KVH, kd = a.kd;
    if (t0 > p) {
        pdl_wait();
        tlm.waited();
        pdl_trigger();
        return;
    }
    const int nt = min(CH, p + 1 - t0);
    const float *kb = a.kc + (size_t)t0 * kd + (size_t)g * HD;
    const float *vb = a.vc + (size_t)t0 * kd + (size_t)g * HD;
    const int nh = min(nt, p - t0);  // rows already in the cache
    for (int i = tid; i < nh * (HD / 4); i += blockDim.x) {
        int t = i / (HD / 4), d4 = i % (HD / 4);
        cp_async16(&ks[t][4 * d4], kb + (size_t)t * kd + 4 * d4);
        cp_async16(&vs[t][4 * d4], vb + (size_t)t * kd + 4 * d4);
    }
    pdl_wait();
    tlm.waited();
    pdl_trigger();
    if (p < 0 || p >= a.max_seq) {
        if (tid == 0 && c == 0 && g == 0) atomicOr(a.err, JDG_ERR_POS);
        cp_async_wait_all();
        return;
    }
    const int half = HD / 2;
    const float *ct = a.rope_cos + (size_t)p * half, *st = a.rope_sin + (size_t)p * half;
    const bool has_p = (p - t0) < CH;
    const int nrot = (hg + (has_p ? 1 : 0)) * half;
    for (int idx = tid; idx < nrot; idx += blockDim.x) {
        int j = idx / half, i = idx % half;
        int i0 = a.rope_norm ? 2 * i : i, i1 = a.rope_norm ? 2 * i + 1 : i + half;
        const float *src = j < hg ? a.qkv + (size_t)(g * hg + j) * HD : a.qkv + a.qd + (size_t)g * HD;
        float x0 = __ldcg(src + i0), x1 = __ldcg(src + i1), cc = ct[i], sn = st[i];
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
        for (int d = tid; d < HD; d += blockDim.x) vs[p - t0][d] = __ldcg(vsrc + d);
    }
    cp_async_wait_all();
    __syncthreads();
    if (has_p) {  // append k (roped) and v at p
        float *kdst = a.kc + (size_t)p * kd + (size_t)g * HD, *vdst = a.vc + (size_t)p * kd + (size_t)g * HD;
        for (int d = tid; d < HD; d += blockDim.x) {
            kdst[d] = ks[p - t0][d];
            vdst[d] = vs[p - t0][d];
        }
    }
    const int ncs = a.max_seq / CH + 1;
    constexpr int E = HD / 32;
    for (int j = warp; j < hg; j += 4) {
        float s[CH / 32];
        float m = -INFINITY;
#pragma unroll
        for (int i = 0; i < CH / 32; i++) {
            int t = lane + 32 * i;
            s[i] = -INFINITY;
            if (t < nt) {
                float d = 0.f;
#pragma unroll
                for (int d4 = 0; d4 < HD / 4; d4++)
                    d = dot4(*reinterpret_cast<const float4 *>(&qs[j][4 * d4]), *reinterpret_cast<const float4 *>(&ks[t][4 * d4]), d);
                float sc = __fmul_rn(d, a.scale);
                if (a.clamp > 0.f) sc = __fmul_rn(a.clamp, tanhf(__fmul_rn(sc, a.inv_clamp)));
                s[i] = sc;
            }
            m = fmaxf(m, s[i]);
        }
        m = warp_max(m);
        float l = 0.f;
#pragma unroll
        for (int i = 0; i < CH / 32; i++) {
            int t = lane + 32 * i;
            float e = t < nt ? expf(s[i] - m) : 0.f;
            ps[j][t] = e;
            l += e;
        }
        l = warp_sum(l);
        __syncwarp();
        float o[E];
#pragma unroll
        for (int q = 0; q < E; q++) o[q] = 0.f;
        for (int t = 0; t < nt; t++) {
            float pt = ps[j][t];
#pragma unroll
            for (int q = 0; q < E; q++) o[q] = fmaf(pt, vs[t][lane * E + q], o[q]);
        }
        float *dst = a.part + ((size_t)(g * hg + j) * ncs + c) * (HD + 2);
#pragma unroll
        for (int q = 0; q < E; q++) dst[lane * E + q] = o[q];
        if (lane == 0) {
            dst[HD] = m;
            dst[HD + 1] = l;
        }
    }
}

template <int HD>
static __global__ __launch_bounds__(128) void k_b1_attn(B1Args a) {
    TlMark tlm(a.tl, a.l * 5 + 1);
    b1_attn_cta<HD>(a, blockIdx.x, blockIdx.y, tlm);
}

// ---------------------------------------------------------------------------------
// WO: att = merge of the attention partials (f_c = e^{m_c-M}/sum l_c e^{m_c-M}), then
// x += Wo . att (janusdoe.c:911-912).  Each CTA also writes, for its 4 rows r, the partial
// sums  sum x_r^2  and  sum (w_vote[e][r] * ffn_norm[r]) * x_r  (e < 16): the FFN RMSNorm
// and the 16 votes in factored form, vote_e = inv * sum (janusdoe.c:915, 795-797).
template <int NV, int HD>
static __global__ __launch_bounds__(128) void k_b1_wo(B1Args a) {
    TlMark tlm(a.tl, a.l * 5 + 2);
    constexpr int CH = kB1Chunk, MAXC = 1024 / CH;
    __shared__ __align__(16) float xs[NV * 128];
    __shared__ float fm[32][MAXC];
    __shared__ float xnew[4];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row = blockIdx.x * 4 + warp;
    float4 w[NV];
    if (row < a.D) {
        const float *wr = a.wo + (size_t)row * a.qd;
#pragma unroll
        for (int j = 0; j < NV; j++) w[j] = ld_stream4(wr + 4 * (lane + 32 * j));
    }
    float wv = 0.f;
    if (threadIdx.x < 64) {
        int e = threadIdx.x >> 2, r = blockIdx.x * 4 + (threadIdx.x & 3);
        if (r < a.D && a.alive[e]) wv = __fmul_rn(a.w_vote[(size_t)e * a.D + r], a.ffn_norm[r]);
    }
    const float xold = row < a.D ? a.x[row] : 0.f;
    const int p = a.pos[0], nc = p / CH + 1, ncs = a.max_seq / CH + 1;
    pdl_wait();
    tlm.waited();
    pdl_trigger();
    float attv[(NV * 128 + 127) / 128];
    float ovs[(NV * 128 + 127) / 128][MAXC];
    // merge weights per head: f_c = e^{m_c - M} / sum_c l_c e^{m_c - M}
    __shared__ float ml[32][MAXC][2];
    {
        float mv[2], lv[2];
        int hh[2], cc[2];
#pragma unroll
        for (int r = 0; r < 2; r++) {
            int idx = threadIdx.x + 128 * r;
            hh[r] = idx / MAXC;
            cc[r] = idx % MAXC;
            bool ok = hh[r] < a.H && cc[r] < nc;
            const float *pp = a.part + ((size_t)hh[r] * ncs + cc[r]) * (HD + 2) + HD;
            mv[r] = ok ? __ldcg(pp) : -INFINITY;
            lv[r] = ok ? __ldcg(pp + 1) : 0.f;
        }
#pragma unroll
        for (int r = 0; r < 2; r++)
            if (hh[r] < 32) {
                ml[hh[r]][cc[r]][0] = mv[r];
                ml[hh[r]][cc[r]][1] = lv[r];
            }
    }
    // att[h*HD + d] = sum_c o_c[d] * f_c   (o_c loaded before the weights f_c are known)
#pragma unroll
    for (int r = 0; r < (NV * 128 + 127) / 128; r++) {
        const int i = threadIdx.x + 128 * r;
        if (i < a.qd) {
            const int h = i / HD, d = i % HD;
            const float *pp = a.part + (size_t)h * ncs * (HD + 2) + d;
            float ov[MAXC];
#pragma unroll
            for (int cc = 0; cc < MAXC; cc++) ov[cc] = cc < nc ? __ldcg(pp + (size_t)cc * (HD + 2)) : 0.f;
            attv[r] = 0.f;
#pragma unroll
            for (int cc = 0; cc < MAXC; cc++) ovs[r][cc] = ov[cc];
        }
    }
    __syncthreads();
    if (threadIdx.x < a.H) {
        const int h = threadIdx.x;
        float M = -INFINITY;
#pragma unroll
        for (int c2 = 0; c2 < MAXC; c2++) M = fmaxf(M, ml[h][c2][0]);
        float S = 0.f, f[MAXC];
#pragma unroll
        for (int c2 = 0; c2 < MAXC; c2++) {
            f[c2] = c2 < nc ? expf(ml[h][c2][0] - M) : 0.f;
            S = fmaf(ml[h][c2][1], f[c2], S);
        }
#pragma unroll
        for (int c2 = 0; c2 < MAXC; c2++) fm[h][c2] = f[c2] / S;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < (NV * 128 + 127) / 128; r++) {
        const int i = threadIdx.x + 128 * r;
        if (i < a.qd) {
            const int h = i / HD;
            float o = 0.f;
#pragma unroll
            for (int cc = 0; cc < MAXC; cc++) o = fmaf(ovs[r][cc], fm[h][cc], o);
            xs[i] = o;
            if (blockIdx.x == 0) a.att[i] = o;
        }
    }
    __syncthreads();
    float xn = 0.f;
    if (row < a.D) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < NV; j++) acc = dot4(w[j], reinterpret_cast<const float4 *>(xs)[lane + 32 * j], acc);
        acc = warp_sum(acc);
        xn = __fadd_rn(xold, acc);
        if (lane == 0) a.x[row] = xn;
    }
    if (lane == 0) xnew[warp] = xn;
    __syncthreads();
    if (threadIdx.x < 64) {
        float pv = __fmul_rn(wv, xnew[threadIdx.x & 3]);
        pv = __fadd_rn(pv, __shfl_xor_sync(0xffffffffu, pv, 1));
        pv = __fadd_rn(pv, __shfl_xor_sync(0xffffffffu, pv, 2));
        if ((threadIdx.x & 3) == 0) a.vpart[(size_t)(threadIdx.x >> 2) * gridDim.x + blockIdx.x] = pv;
    }
    if (threadIdx.x == 64) {
        float ss = 0.f;
        for (int q = 0; q < 4; q++) ss = __fadd_rn(ss, __fmul_rn(xnew[q], xnew[q]));
        a.vpart[(size_t)16 * gridDim.x + blockIdx.x] = ss;
    }
    // the last CTA reduces the partials and runs the parliament election for this layer
    if (!last_cta(a.tickets + 32, gridDim.x)) return;
    __shared__ ElectOut eo;
    b1_elect(a, eo, __ldcg(a.consensus + a.l));
    if (threadIdx.x < kMaxE) {
        const int q = threadIdx.x, k = eo.k;
        a.sel[q] = eo.sel[q];
        a.selw[q] = eo.w[q];
        a.sel_gu[q] = q < k ? a.gu_tab[eo.sel[q]] : nullptr;
        a.sel_dn[q] = q < k ? a.dn_tab[eo.sel[q]] : nullptr;
        a.tr_sel[(size_t)a.l * kMaxE + q] = eo.sel[q];
        a.tr_w[(size_t)a.l * kMaxE + q] = eo.w[q];
    }
    if (threadIdx.x == 0) {
        a.kcnt[0] = eo.k;
        a.tr_k[a.l] = eo.k;
        a.tr_ema[a.l] = eo.ema;
        a.consensus[a.l] = eo.ema;
        *a.ffn_inv = eo.inv;
        atomicAdd(a.stats, (unsigned long long)eo.k);
        a.tickets[32] = 0;
    }
}

// ---------------------------------------------------------------------------------
// FFN1: every CTA runs the election (b1_elect); CTA 0 publishes it (k, slots, weights,
// trace, the EMA to commit one kernel later); each CTA warms L2 with its slice of the
// elected experts' down rows; then h_ki[i] = silu(Wg_e[i].xb) * (Wu_e[i].xb)
// (janusdoe.c:921-925), xb = rmsnorm(x, ffn_norm) with the election's norm factor.
// Warps walk the (ki, i) hidden units with a stride of all warps of the grid; rows
// (2i, 2i+1) of the interleaved gate/up matrix.
template <int NV>
static __global__ __launch_bounds__(128) void k_b1_ffn1(B1Args a) {
    TlMark tlm(a.tl, a.l * 5 + 3);
    __shared__ __align__(16) float xs[NV * 128];
    __shared__ const float *gu_s[kMaxE];
    __shared__ const float *dn_s[kMaxE];
    __shared__ int k_s;
    __shared__ __align__(16) float fnw[NV * 128];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < a.D / 4; i += 128)
        reinterpret_cast<float4 *>(fnw)[i] = reinterpret_cast<const float4 *>(a.ffn_norm)[i];
    pdl_wait();
    tlm.waited();
    pdl_trigger();
    float4 xr[(NV + 3) / 4];
#pragma unroll
    for (int j = 0; j < (NV + 3) / 4; j++) {
        int i = threadIdx.x + 128 * j;
        if (i < a.D / 4) xr[j] = __ldcg(reinterpret_cast<const float4 *>(a.x) + i);
    }
    const float inv = __ldcg(a.ffn_inv);
    if (threadIdx.x < kMaxE) {
        gu_s[threadIdx.x] = (const float *)__ldcg((const unsigned long long *)(a.sel_gu + threadIdx.x));
        dn_s[threadIdx.x] = (const float *)__ldcg((const unsigned long long *)(a.sel_dn + threadIdx.x));
    }
    if (threadIdx.x == 0) k_s = __ldcg(a.kcnt);
    __syncthreads();
    const int k = k_s;
    // warm L2 with this CTA's share of the elected down matrices (read by FFN2)
    {
        const size_t lines = (size_t)a.D * a.hidden * 4 / 128;
        const size_t per = (lines + gridDim.x - 1) / gridDim.x, l0 = per * blockIdx.x;
        for (int q = 0; q < k; q++) {
            const char *base = reinterpret_cast<const char *>(dn_s[q]);
            for (size_t li = l0 + threadIdx.x; li < l0 + per && li < lines; li += 128) prefetch_l2(base + li * 128);
        }
    }
#pragma unroll
    for (int j = 0; j < (NV + 3) / 4; j++) {
        int i = threadIdx.x + 128 * j;
        if (i < a.D / 4) {
            float4 f = reinterpret_cast<const float4 *>(fnw)[i], v = xr[j];
            v.x = __fmul_rn(__fmul_rn(v.x, inv), f.x);
            v.y = __fmul_rn(__fmul_rn(v.y, inv), f.y);
            v.z = __fmul_rn(__fmul_rn(v.z, inv), f.z);
            v.w = __fmul_rn(__fmul_rn(v.w, inv), f.w);
            reinterpret_cast<float4 *>(xs)[i] = v;
        }
    }
    __syncthreads();
    const int nunits = k * a.hidden, gw = gridDim.x * 4;
    // two units in flight per warp: the next unit's rows load while this one computes
    float4 ga[NV], ua[NV], gb[NV], ub[NV];
    auto load_unit = [&](int uu, float4 (&g4)[NV], float4 (&u4)[NV]) {
        if (uu >= nunits) return;
        const int ki = uu / a.hidden, i = uu - ki * a.hidden;
        const float *g = gu_s[ki] + (size_t)(2 * i) * a.D, *up = g + a.D;
#pragma unroll
        for (int j = 0; j < NV; j++) {
            g4[j] = ld_stream4(g + 4 * (lane + 32 * j));
            u4[j] = ld_stream4(up + 4 * (lane + 32 * j));
        }
    };
    auto compute_unit = [&](int uu, const float4 (&g4)[NV], const float4 (&u4)[NV]) {
        float ag = 0.f, au = 0.f;
#pragma unroll
        for (int j = 0; j < NV; j++) {
            float4 xv = reinterpret_cast<const float4 *>(xs)[lane + 32 * j];
            ag = dot4(g4[j], xv, ag);
            au = dot4(u4[j], xv, au);
        }
        ag = warp_sum(ag);
        au = warp_sum(au);
        const int ki = uu / a.hidden, i = uu - ki * a.hidden;
        if (lane == 0) a.hbuf[(size_t)ki * a.hidden + i] = __fmul_rn(silu_ref(ag), au);
    };
    int u = blockIdx.x * 4 + warp;
    load_unit(u, ga, ua);
    while (u < nunits) {
        load_unit(u + gw, gb, ub);
        compute_unit(u, ga, ua);
        u += gw;
        if (u >= nunits) break;
        load_unit(u + gw, ga, ua);
        compute_unit(u, gb, ub);
        u += gw;
    }
}

// ---------------------------------------------------------------------------------
// FFN2: y_ki[r] = Wd_e[r] . h_ki for the elected experts (janusdoe.c:926); the weighted
// sum and residual add happen in the next kernel's prologue.  grid (D/4, kmax).
template <int NH>
static __global__ __launch_bounds__(128) void k_b1_ffn2(B1Args a) {
    TlMark tlm(a.tl, a.l * 5 + 4);
    __shared__ __align__(16) float hs[NH * 128];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ki = blockIdx.y, rb = blockIdx.x, r = rb * 4 + warp;
    // the election was published by WO (two kernels back): load the down rows now
    const int k = __ldcg(a.kcnt);
    const float *W = ki < k ? (const float *)__ldcg((const unsigned long long *)(a.sel_dn + ki)) : nullptr;
    float4 w[NH];
    if (W && r < a.D) {
        const float *wr = W + (size_t)r * a.hidden;
#pragma unroll
        for (int j = 0; j < NH; j++) w[j] = ld_stream4(wr + 4 * (lane + 32 * j));
    }
    pdl_wait();
    tlm.waited();
    pdl_trigger();
    if (ki >= k) return;
    if (W == nullptr && threadIdx.x == 0) atomicOr(a.err, JDG_ERR_ROUTE);
    vec_to_smem<(NH + 3) / 4>(hs, a.hbuf + (size_t)ki * a.hidden, a.hidden / 4);
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
    // the last CTA of this row block adds sum_ki w_ki * y_ki in election order
    // (janusdoe.c:927-929); x is updated in place, rows are owned by one CTA each
    if (!last_cta(a.tickets + 64 + rb, k)) return;
    if (threadIdx.x < 4) {
        const int rr = rb * 4 + threadIdx.x;
        if (rr < a.D) {  // every operand loaded before the ordered sum
            const float xo = a.x[rr];
            float wv[kMaxE], yv[kMaxE];
#pragma unroll
            for (int q = 0; q < kMaxE; q++) {
                wv[q] = q < k ? __ldcg(a.selw + q) : 0.f;
                yv[q] = q < k ? __ldcg(a.ybuf + (size_t)q * a.D + rr) : 0.f;
            }
            float eo = 0.f;
#pragma unroll
            for (int q = 0; q < kMaxE; q++)
                if (q < k) eo = __fadd_rn(eo, __fmul_rn(wv[q], yv[q]));
            a.x[rr] = __fadd_rn(xo, eo);
        }
    }
    if (threadIdx.x == 0) a.tickets[64 + rb] = 0;
}

// ---------------------------------------------------------------------------------
// LMHEAD: x += last layer's expert outputs, logits = Wout . rmsnorm(x, output_norm)
// (janusdoe.c:931-932).  Per-CTA argmax partials; with greedy_pick the last CTA takes the
// first-index maximum (janusdoe.c:3637) or the prompt's next id and advances tok/pos/history.
template <int NV>
static __global__ __launch_bounds__(128) void k_b1_lmhead(B1Args a) {
    TlMark tlm(a.tl, a.L * 5);
    __shared__ __align__(16) float xs[NV * 128];
    __shared__ float red[32];
    __shared__ float bv_s[4];
    __shared__ int bi_s[4];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // warp-stride loop over row pairs, two pairs in flight
    const int gw = gridDim.x * 4;
    const int npair = (a.V + 1) / 2;
    float4 wa[2][NV], wb[2][NV];
    auto load_pair = [&](int pr, float4 (&w4)[2][NV]) {
        if (pr >= npair) return;
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const int row = 2 * pr + r;
            if (row < a.V) {
                const float *wr = a.output + (size_t)row * a.D;
#pragma unroll
                for (int j = 0; j < NV; j++) w4[r][j] = ld_stream4(wr + 4 * (lane + 32 * j));
            }
        }
    };
    int pr = blockIdx.x * 4 + warp;
    load_pair(pr, wa);
    pdl_wait();
    tlm.waited();
    pdl_trigger();
    b1_load_x<NV>(a, xs);
    __syncthreads();
    float ss = 0.f;
    for (int i = threadIdx.x; i < a.D / 4; i += blockDim.x) {
        float4 v = reinterpret_cast<const float4 *>(xs)[i];
        ss = dot4(v, v, ss);
    }
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)a.D + a.eps);
    for (int i = threadIdx.x; i < a.D; i += 128) xs[i] = __fmul_rn(__fmul_rn(xs[i], inv), a.output_norm[i]);
    __syncthreads();
    float val = -INFINITY;
    int vi = 0x7fffffff;
    auto compute_pair = [&](int p2, const float4 (&w4)[2][NV]) {
        float acc[2] = {0.f, 0.f};
#pragma unroll
        for (int j = 0; j < NV; j++) {
            float4 xv = reinterpret_cast<const float4 *>(xs)[lane + 32 * j];
#pragma unroll
            for (int r = 0; r < 2; r++) acc[r] = dot4(w4[r][j], xv, acc[r]);
        }
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const float v = warp_sum(acc[r]);
            const int row = 2 * p2 + r;
            if (row < a.V) {
                if (lane == 0) a.logits[row] = v;
                if (v > val) {  // rows visited in increasing order per warp: first max kept
                    val = v;
                    vi = row;
                }
            }
        }
    };
    while (pr < npair) {
        load_pair(pr + gw, wb);
        compute_pair(pr, wa);
        pr += gw;
        if (pr >= npair) break;
        load_pair(pr + gw, wa);
        compute_pair(pr, wb);
        pr += gw;
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
    for (int q0 = 0; q0 < (int)gridDim.x; q0 += 128 * 16) {
        float vv[16];
        int ii[16];
#pragma unroll
        for (int j = 0; j < 16; j++) {
            int q = q0 + threadIdx.x + 128 * j;
            vv[j] = q < (int)gridDim.x ? __ldcg(a.amax_v + q) : -INFINITY;
            ii[j] = q < (int)gridDim.x ? __ldcg(a.amax_i + q) : 0x7fffffff;
        }
#pragma unroll
        for (int j = 0; j < 16; j++)
            if (vv[j] > bv || (vv[j] == bv && ii[j] < bi)) {
                bv = vv[j];
                bi = ii[j];
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


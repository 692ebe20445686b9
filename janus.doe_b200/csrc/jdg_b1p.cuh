// jdg_b1p.cuh — the batch-1 own-model decode step (forward_token + greedy pick,
// janusdoe.c:879-934, 3637) as ONE persistent kernel.
//
// One CTA per SM, all resident (cooperative launch), 256 threads.  Per layer five phases,
// separated by grid barriers (a release/acquire counter with a bounded wait):
//   P1  x (layer 0: tok_emb[tok]) -> RMSNorm -> this CTA's q/k/v rows
//   P2  attention, one item (KV head g, 64-position chunk c) per CTA: RoPE (NeoX halves),
//       KV append, scores with the clamp*tanh(s/clamp) of janusdoe.c:906, chunk softmax
//       partials (o, m, l)
//   P3  every CTA merges the partials into att; this CTA's Wo rows: x += Wo.att; partial
//       votes  sum_r (w_vote[e][r]*ffn_norm[r]) * x_r  and  sum_r x_r^2  of its rows
//   P4  every CTA reduces the partials in the same fixed order and runs the same election
//       (janusdoe.c:779-838); all warps of the grid stream the elected experts' gate/up
//       rows: h = silu(g.xb) * (u.xb)
//   P5  this CTA's rows of the elected experts' down projections, combined in election
//       order into x (janusdoe.c:926-929)
// then the LM head (final RMSNorm, logits, first-index argmax, the last CTA advances the
// token / position / history).
// Weights whose addresses do not depend on the step's data — the next layer's q/k/v rows
// and Wo rows of this CTA, the KV history of its attention item — are copied into shared
// memory by the bulk-copy engine while earlier phases run, so the latency-bound phases
// P1-P3 read them from shared memory; P4 warms L2 with the down rows P5 reads (and, in
// the last layer, the LM head rows).
#pragma once
#include "jdg_async.cuh"
#include "jdg_kernels.cuh"

namespace jdg {

constexpr int kPThreads = 256, kPWarps = kPThreads / 32;
constexpr int kPChunk = 64;   // attention positions per item
constexpr int kPHD = 64;      // head dimension of the own model
constexpr int kPKRow = kPHD + 4;  // padded K/V row in shared memory (conflict-free float4)
constexpr int kPMaxHG = 8;    // query heads per KV head

// Per-layer parameter block in device memory (built at upload), staged into shared memory
// one layer ahead: [B1PLayer, padded to kPParHdr bytes][attn_norm D][ffn_norm D][wvn D x 16]
// with wvn[r][e] = w_vote[e][r] * ffn_norm[r] (0 for dead slots), the factored vote rows.
struct B1PLayer {
    const float *wqkv, *wo;
    const float *gu[kMaxE];   // gate/up rows interleaved [2*hidden][D] of alive slots, else null
    const float *dn[kMaxE];   // down [D][hidden]
    unsigned alive;           // bit e: slot e alive
    float temperature;
};
constexpr int kPParHdr = 320;
static_assert(sizeof(B1PLayer) <= kPParHdr, "layer header");
__host__ __device__ inline size_t b1p_par_stride(int D) { return kPParHdr + (size_t)18 * D * 4; }

struct B1PArgs {
    const char *layers;      // L parameter blocks of b1p_par_stride(D) bytes
    const float *tok_emb, *output, *output_norm, *rope_cos, *rope_sin;
    int V, D, H, KVH, hidden, qkvd, max_seq, L, kmax, nch_max;
    float eps, scale, clamp, inv_clamp;
    const int *tok;
    int *pos;
    float *x, *qkv, *part, *vpart, *hbuf, *logits, *kc, *vc, *consensus;
    int *tr_k, *tr_sel;
    float *tr_w, *tr_ema;
    unsigned *bar;      // grid barrier counter, zeroed before every launch
    unsigned *ticket;   // LM-head last-CTA counter (reset by the last CTA)
    float *amax_v;
    int *amax_i;
    unsigned long long *stats;
    int *tok_out, *plen, *prompt, *hist, *hist_n, *next_out;
    int Hmax, greedy_pick;
    int *err;
    unsigned long long *tl;  // optional phase timeline [slot][3]
    int rq, rd;              // q/k/v rows and model rows per CTA (at most)
};

// Shared-memory carve of the persistent step (floats; every piece 16-byte aligned).
struct B1PSmem {
    int wqkv, wo, k, v, x, att, h, q, p, po, ml, fm, y, xr, par0, par1, onorm, rope, total;
};
__host__ __device__ inline B1PSmem b1p_smem(int D, int H, int hidden, int kmax, int nch_max, int rq, int rd) {
    B1PSmem s;
    int o = 0;
    auto take = [&](int n) { int r = o; o += (n + 3) & ~3; return r; };
    s.wqkv = take(rq * D);
    s.wo = take(rd * D);
    s.k = take(kPChunk * kPKRow);
    s.v = take(kPChunk * kPKRow);
    s.x = take(D);
    s.att = take(D);
    s.h = take(kmax * hidden);
    s.q = take(kPMaxHG * kPHD);
    s.p = take(kPMaxHG * kPChunk);
    s.po = take(4 * kPMaxHG * kPHD);
    s.ml = take(H * nch_max * 2);
    s.fm = take(H * nch_max);
    s.y = take(rd * kMaxE);
    s.xr = take(rd);
    s.par0 = take(kPParHdr / 4 + 2 * D + 16 * rd);
    s.par1 = take(kPParHdr / 4 + 2 * D + 16 * rd);
    s.onorm = take(D);
    s.rope = take(kPHD);
    s.total = o;
    return s;
}

__device__ __forceinline__ unsigned long long p_gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

constexpr unsigned long long kPWaitNs = 200ull * 1000 * 1000;  // 200 ms: any wait longer is an error

__device__ __forceinline__ int p_err_now(const int *err) {
    int e;
    asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(e) : "l"(err) : "memory");
    return e;
}

// Grid barrier: every CTA adds one to the counter (release), then waits (acquire) for the
// count of this barrier generation.  The wait gives up after kPWaitNs of wall time, or as
// soon as another CTA has recorded a timeout, and then reports false.
__device__ __forceinline__ bool p_grid_sync(const B1PArgs &a, unsigned &gen, int *s_flag, int slot) {
    gen += gridDim.x;
    __syncthreads();
    if (threadIdx.x == 0) {
        if (a.tl) atomicMax(a.tl + 3 * slot + 2, p_gtimer());
        __threadfence();
        atomicAdd(a.bar, 1u);
        int ok = 1;
        const unsigned long long t0 = p_gtimer();
        for (int it = 0;; it++) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a.bar) : "memory");
            if (v >= gen) break;
            if ((it & 31) == 31) {
                if (p_err_now(a.err) & JDG_ERR_TIMEOUT) { ok = 0; break; }
                if (p_gtimer() - t0 > kPWaitNs) {
                    atomicOr(a.err, JDG_ERR_TIMEOUT);
                    ok = 0;
                    break;
                }
            }
        }
        if (a.tl) {  // the next phase starts here in this CTA
            const unsigned long long t = p_gtimer();
            atomicMin(a.tl + 3 * (slot + 1), t);
            atomicMax(a.tl + 3 * (256 + slot + 1) + 2, t);
        }
        *s_flag = ok;
    }
    __syncthreads();
    return *s_flag != 0;
}

// L2 prefetch of [p, p + bytes) by the bulk-copy engine (no shared memory involved), split
// into pieces of at most 64 KB with 16-byte granularity.
__device__ __forceinline__ void p_prefetch_range(const void *p, size_t bytes) {
    const char *c = reinterpret_cast<const char *>(p);
    while (bytes >= 16) {
        const uint32_t n = (uint32_t)(bytes > 65536 ? 65536 : bytes) & ~15u;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(c), "r"(n) : "memory");
        c += n;
        bytes -= n;
    }
}
// This CTA's share (1/G, by blockIdx) of [p, p + bytes) prefetched into L2.
__device__ __forceinline__ void p_prefetch_share(const void *p, size_t bytes) {
    const size_t per = ((bytes + gridDim.x - 1) / gridDim.x + 15) & ~(size_t)15;
    const size_t off = per * blockIdx.x;
    if (off < bytes) p_prefetch_range(reinterpret_cast<const char *>(p) + off, off + per > bytes ? bytes - off : per);
}

// Wait for phase `parity` of a shared-memory mbarrier (bulk copies landing) with the same
// wall-time limit; false when it ran out or (err given) another CTA recorded a timeout.
__device__ __forceinline__ bool p_mbar_wait(uint64_t *bar, uint32_t parity, const int *err) {
    const unsigned long long t0 = p_gtimer();
    for (int it = 0;; it++) {
        uint32_t done;
        asm volatile("{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                     : "=r"(done)
                     : "r"(smem_u32(bar)), "r"(parity)
                     : "memory");
        if (done) return true;
        if ((it & 63) == 63 && ((err && (p_err_now(err) & JDG_ERR_TIMEOUT)) || p_gtimer() - t0 > kPWaitNs))
            return false;
    }
}

// The election of janusdoe.c:779-838 on warp 0 from the reduced totals (tot[e] = sum of
// the partial votes of slot e, tot[16] = sum x^2 over the model rows).
struct PElect {
    int k;
    int sel[kMaxE];
    float w[kMaxE];
    float ema, inv;
};
__device__ __forceinline__ void p_elect_warp0(const float *tot, unsigned am, float cons_in, float temperature, int D,
                                              float eps, PElect &eo) {
    const int lane = threadIdx.x & 31;
    const float inv = 1.0f / sqrtf(tot[16] / (float)D + eps);
    float v[kMaxE];
#pragma unroll
    for (int e = 0; e < kMaxE; e++) v[e] = __fmul_rn(inv, tot[e]);  // dot + 0.1f * 0 (harmonic state is zero)
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
                const float dd = __fsub_rn(v[e], mean);
                var = __fadd_rn(var, __fmul_rn(dd, dd));
            }
        var = var / (float)na;
        const float cs = fminf(1.0f, sqrtf(__fadd_rn(var, 1e-8f)) / __fadd_rn(fabsf(mean), 1.0f));
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
        const float temp = temperature > 0.05f ? temperature : 1.0f;
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
    __syncwarp();
}

// rows [r0, r1) of a matrix with n rows split over the grid: CTA c owns [c*n/G, (c+1)*n/G)
__device__ __forceinline__ void p_rows(int n, int &r0, int &r1) {
    r0 = (int)((long)blockIdx.x * n / gridDim.x);
    r1 = (int)((long)(blockIdx.x + 1) * n / gridDim.x);
}

// Copy n float4 from global (L2) to shared memory, BATCH loads in flight per thread.
template <int BATCH>
__device__ __forceinline__ void p_g2s(float4 *dst, const float4 *src, int n) {
    for (int base = 0; base < n; base += BATCH * kPThreads) {
        float4 r[BATCH];
#pragma unroll
        for (int j = 0; j < BATCH; j++) {
            const int i = base + threadIdx.x + j * kPThreads;
            if (i < n) r[j] = __ldcg(src + i);
        }
#pragma unroll
        for (int j = 0; j < BATCH; j++) {
            const int i = base + threadIdx.x + j * kPThreads;
            if (i < n) dst[i] = r[j];
        }
    }
}

// NV = D/128 float4 per lane for a D-long row, NH = hidden/128.
template <int NV, int NH>
static __global__ __launch_bounds__(kPThreads, 1) void k_b1_step(B1PArgs a) {
    extern __shared__ __align__(128) float sm[];
    // 0: q/k/v rows, 1: KV history, 2: Wo rows, 3/4: layer parameters (by layer parity),
    // 5: output norm + RoPE row
    __shared__ __align__(8) uint64_t mb[6];
    __shared__ float tot[17];
    __shared__ float ema_s[JD_MAX_LAYERS];
    __shared__ PElect eo;
    __shared__ float red[32];
    __shared__ int s_flag;
    __shared__ float bv_s[kPWarps];
    __shared__ int bi_s[kPWarps];
    __shared__ const float *s_gub[kMaxE];  // gate/up matrices of the elected experts, in election order
    const int D = a.D, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, hg = a.H / a.KVH, kd = a.KVH * kPHD;
    const B1PSmem L = b1p_smem(D, a.H, a.hidden, a.kmax, a.nch_max, a.rq, a.rd);
    float *s_wqkv = sm + L.wqkv, *s_wo = sm + L.wo, *s_k = sm + L.k, *s_v = sm + L.v, *s_x = sm + L.x;
    float *s_att = sm + L.att, *s_h = sm + L.h, *s_q = sm + L.q, *s_p = sm + L.p, *s_ml = sm + L.ml;
    float *s_po = sm + L.po;
    float *s_fm = sm + L.fm, *s_y = sm + L.y, *s_xr = sm + L.xr, *s_onorm = sm + L.onorm, *s_rope = sm + L.rope;
    float *s_par[2] = {sm + L.par0, sm + L.par1};

    const int p = __ldcg(a.pos);
    if (p < 0 || p >= a.max_seq) {
        if (tid == 0 && blockIdx.x == 0) atomicOr(a.err, JDG_ERR_POS);
        return;  // every CTA reads the same position and leaves before any barrier
    }
    int tk = __ldcg(a.tok);
    if (tk < 0 || tk >= a.V) {
        if (tid == 0 && blockIdx.x == 0) atomicOr(a.err, JDG_ERR_TOKEN);
        tk = 0;
    }
    int q0, q1, d0, d1;
    p_rows(a.qkvd, q0, q1);
    p_rows(D, d0, d1);
    const int nq = q1 - q0, nr = d1 - d0;
    const int nch = p / kPChunk + 1;
    const int item = blockIdx.x, ich = item / a.KVH, ig = item % a.KVH;
    const bool has_item = ich < nch;
    const int it0 = ich * kPChunk;
    const int i_nt = has_item ? min(kPChunk, p + 1 - it0) : 0;
    const int i_nh = has_item ? min(i_nt, p - it0) : 0;  // history rows already in the cache
    const size_t pstride = b1p_par_stride(D);
    unsigned gen = 0, ph[6] = {0, 0, 0, 0, 0, 0}, pend = 0;  // mbarrier phases; bulk copies not yet waited for

    if (tid < a.L) ema_s[tid] = __ldcg(a.consensus + tid);
    if (tid == 0) {
        for (int i = 0; i < 6; i++) mbar_init(&mb[i], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // bulk copies (one elected thread; warp 0 for the KV rows)
    auto stage_qkv = [&](int l) {
        pend |= 1u << 0;
        if (tid == 0) {
            const uint32_t bytes = (uint32_t)nq * D * 4;
            const B1PLayer *hdr = reinterpret_cast<const B1PLayer *>(a.layers + (size_t)l * pstride);
            mbar_expect_tx(&mb[0], bytes);
            if (bytes) bulk_g2s(s_wqkv, hdr->wqkv + (size_t)q0 * D, bytes, &mb[0]);
        }
    };
    auto stage_wo = [&](int l) {
        pend |= 1u << 2;
        if (tid == 0) {
            const uint32_t bytes = (uint32_t)nr * D * 4;
            const B1PLayer *hdr = reinterpret_cast<const B1PLayer *>(a.layers + (size_t)l * pstride);
            mbar_expect_tx(&mb[2], bytes);
            if (bytes) bulk_g2s(s_wo, hdr->wo + (size_t)d0 * D, bytes, &mb[2]);
        }
    };
    auto stage_kv = [&](int l) {
        if (!has_item) return;
        pend |= 1u << 1;
        if (warp != 0) return;
        if (lane == 0) mbar_expect_tx(&mb[1], (uint32_t)i_nh * 2 * kPHD * 4);
        __syncwarp();
        const float *kb = a.kc + (size_t)l * a.max_seq * kd + (size_t)it0 * kd + (size_t)ig * kPHD;
        const float *vb = a.vc + (size_t)l * a.max_seq * kd + (size_t)it0 * kd + (size_t)ig * kPHD;
        for (int t = lane; t < i_nh; t += 32) {
            bulk_g2s(s_k + t * kPKRow, kb + (size_t)t * kd, kPHD * 4, &mb[1]);
            bulk_g2s(s_v + t * kPKRow, vb + (size_t)t * kd, kPHD * 4, &mb[1]);
        }
    };
    // layer l's header, norms and this CTA's factored vote rows into s_par[l & 1]
    auto stage_par = [&](int l) {
        pend |= 1u << (3 + (l & 1));
        if (tid == 0) {
            const char *blk = a.layers + (size_t)l * pstride;
            const uint32_t b0 = kPParHdr + 2u * D * 4, b1 = (uint32_t)nr * 16 * 4;
            uint64_t *bar = &mb[3 + (l & 1)];
            mbar_expect_tx(bar, b0 + b1);
            bulk_g2s(s_par[l & 1], blk, b0, bar);
            if (b1) bulk_g2s(s_par[l & 1] + b0 / 4, blk + b0 + (size_t)d0 * 16 * 4, b1, bar);
        }
    };
    auto release_and = [&](auto &&issue) {  // generic reads of a buffer done -> async refill
        fence_proxy_async_smem();
        __syncthreads();
        issue();
    };
    auto wait_bar = [&](int i) -> bool {
        const bool ok = p_mbar_wait(&mb[i], ph[i], a.err);
        ph[i] ^= 1u;
        pend &= ~(1u << i);
        if (!ok && lane == 0) atomicOr(a.err, JDG_ERR_TIMEOUT);
        return ok;
    };
    // error exit: wait (bounded by time alone) for this CTA's bulk copies still in flight
    auto drain = [&]() {
        for (int i = 0; i < 6; i++)
            if (pend & (1u << i)) p_mbar_wait(&mb[i], ph[i], nullptr);
    };
    stage_par(0);
    stage_qkv(0);
    stage_kv(0);
    stage_wo(0);
    pend |= 1u << 5;
    if (tid == 0) {  // the output norm and the RoPE row of this position
        mbar_expect_tx(&mb[5], (uint32_t)(D + kPHD) * 4);
        bulk_g2s(s_onorm, a.output_norm, D * 4, &mb[5]);
        bulk_g2s(s_rope, a.rope_cos + (size_t)p * (kPHD / 2), kPHD / 2 * 4, &mb[5]);
        bulk_g2s(s_rope + kPHD / 2, a.rope_sin + (size_t)p * (kPHD / 2), kPHD / 2 * 4, &mb[5]);
    }
    const size_t gu_bytes = (size_t)2 * a.hidden * D * 4;
    if (tid < kMaxE) {  // layer 0's gate/up matrices of every alive expert, this CTA's share, into L2
        const float *g = reinterpret_cast<const B1PLayer *>(a.layers)->gu[tid];
        if (g) p_prefetch_share(g, gu_bytes);
    }
    if (a.tl && tid == 0) {
        const unsigned long long t = p_gtimer();
        atomicMin(a.tl, t);
        atomicMin(a.tl + 3, t);
        atomicMax(a.tl + 3 * 257 + 2, t);
    }
    bool misc_ready = false;
    bool par_ready = false;  // the next layer's parameters were already waited for (in P5)
    // fine timeline of CTA 0 (debug): slot 300 + 8*layer + i
    auto mark = [&](int l, int i) {
        if (a.tl && blockIdx.x == 0 && tid == 0 && l < 26) a.tl[3 * (300 + 8 * l + i)] = p_gtimer();
    };

    for (int l = 0; l < a.L; l++) {
        const int slot = 1 + 5 * l;
        if (l + 1 < a.L) stage_par(l + 1);  // its buffer was last read by layer l-1
        if (!par_ready) wait_bar(3 + (l & 1));
        par_ready = false;
        const float *par = s_par[l & 1];
        const B1PLayer &ly = *reinterpret_cast<const B1PLayer *>(par);
        // the HBM is idle in the latency-bound phases P1-P3: bring this layer's gate/up
        // matrices of every alive expert (the election is not known yet) into L2 for P4;
        // in the last layer also the LM head
        if (l > 0 && tid < kMaxE && ly.gu[tid]) p_prefetch_share(ly.gu[tid], gu_bytes);
        if (l + 1 == a.L && tid == kMaxE) p_prefetch_share(a.output, (size_t)a.V * D * 4);
        mark(l, 0);
        const float *attn_norm = par + kPParHdr / 4, *ffn_norm = attn_norm + D, *wvn = ffn_norm + D;
        // ---------------- P1: RMSNorm + q/k/v rows ----------------
        {
            const float *src = l == 0 ? a.tok_emb + (size_t)tk * D : a.x;
            p_g2s<4>(reinterpret_cast<float4 *>(s_x), reinterpret_cast<const float4 *>(src), D / 4);
            __syncthreads();
            if (l == 0 && blockIdx.x == 0)
                for (int i = tid; i < D / 4; i += kPThreads)
                    reinterpret_cast<float4 *>(a.x)[i] = reinterpret_cast<const float4 *>(s_x)[i];
            if (tid < nr) s_xr[tid] = s_x[d0 + tid];  // residual of this CTA's model rows
            float ss = 0.f;
            for (int i = tid; i < D / 4; i += kPThreads) {
                const float4 v = reinterpret_cast<const float4 *>(s_x)[i];
                ss = dot4(v, v, ss);
            }
            ss = block_sum(ss, red);
            const float inv = 1.0f / sqrtf(ss / (float)D + a.eps);
            for (int i = tid; i < D; i += kPThreads) s_x[i] = __fmul_rn(__fmul_rn(s_x[i], inv), attn_norm[i]);
            __syncthreads();
            mark(l, 1);
            wait_bar(0);
            for (int rr = warp; rr < nq; rr += kPWarps) {
                const float *wr = s_wqkv + (size_t)rr * D;
                float acc = 0.f;
#pragma unroll
                for (int j = 0; j < NV; j++) {
                    const int i4 = lane + 32 * j;
                    acc = dot4(reinterpret_cast<const float4 *>(wr)[i4], reinterpret_cast<const float4 *>(s_x)[i4], acc);
                }
                acc = warp_sum(acc);
                if (lane == 0) a.qkv[q0 + rr] = acc;
            }
            if (l + 1 < a.L) release_and([&] { stage_qkv(l + 1); });
        }
        if (!p_grid_sync(a, gen, &s_flag, slot)) { drain(); return; }
        // ---------------- P2: attention item ----------------
        if (has_item) {
            if (!misc_ready) {
                wait_bar(5);
                misc_ready = true;
            }
            float *kdst_l = a.kc + (size_t)l * a.max_seq * kd, *vdst_l = a.vc + (size_t)l * a.max_seq * kd;
            const int half = kPHD / 2;
            const bool has_p = p - it0 < kPChunk;
            const int nrot = (hg + (has_p ? 1 : 0)) * half;
            for (int idx = tid; idx < nrot; idx += kPThreads) {
                const int j = idx / half, i = idx % half;
                const float *src = j < hg ? a.qkv + (size_t)(ig * hg + j) * kPHD : a.qkv + D + (size_t)ig * kPHD;
                const float x0 = __ldcg(src + i), x1 = __ldcg(src + i + half), cc = s_rope[i], sn = s_rope[half + i];
                const float y0 = __fsub_rn(__fmul_rn(x0, cc), __fmul_rn(x1, sn));
                const float y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cc));
                if (j < hg) {
                    s_q[j * kPHD + i] = y0;
                    s_q[j * kPHD + i + half] = y1;
                } else {
                    s_k[(p - it0) * kPKRow + i] = y0;
                    s_k[(p - it0) * kPKRow + i + half] = y1;
                }
            }
            if (has_p && tid < kPHD) s_v[(p - it0) * kPKRow + tid] = __ldcg(a.qkv + D + kd + (size_t)ig * kPHD + tid);
            wait_bar(1);
            __syncthreads();
            mark(l, 2);
            if (has_p && tid < kPHD) {  // append k (roped) and v at p
                kdst_l[(size_t)p * kd + (size_t)ig * kPHD + tid] = s_k[(p - it0) * kPKRow + tid];
                vdst_l[(size_t)p * kd + (size_t)ig * kPHD + tid] = s_v[(p - it0) * kPKRow + tid];
            }
            for (int idx = tid; idx < hg * kPChunk; idx += kPThreads) {  // scores: (head j, position t)
                const int j = idx / kPChunk, t = idx % kPChunk;
                if (t < i_nt) {
                    float d = 0.f;
#pragma unroll
                    for (int d4 = 0; d4 < kPHD / 4; d4++)
                        d = dot4(reinterpret_cast<const float4 *>(s_q + j * kPHD)[d4],
                                 reinterpret_cast<const float4 *>(s_k + t * kPKRow)[d4], d);
                    float sc = __fmul_rn(d, a.scale);
                    if (a.clamp > 0.f) sc = __fmul_rn(a.clamp, tanhf(__fmul_rn(sc, a.inv_clamp)));
                    s_p[j * kPChunk + t] = sc;
                }
            }
            __syncthreads();
            mark(l, 3);
            for (int j = warp; j < hg; j += kPWarps) {  // chunk softmax of head j
                const float s0 = lane < i_nt ? s_p[j * kPChunk + lane] : -INFINITY;
                const float s1 = lane + 32 < i_nt ? s_p[j * kPChunk + lane + 32] : -INFINITY;
                const float m = warp_max(fmaxf(s0, s1));
                const float e0 = lane < i_nt ? expf(s0 - m) : 0.f, e1 = lane + 32 < i_nt ? expf(s1 - m) : 0.f;
                s_p[j * kPChunk + lane] = e0;
                s_p[j * kPChunk + lane + 32] = e1;
                const float lsum = warp_sum(e0 + e1);
                if (lane == 0) {
                    float *dst = a.part + ((size_t)(ig * hg + j) * a.nch_max + ich) * (kPHD + 2);
                    dst[kPHD] = m;
                    dst[kPHD + 1] = lsum;
                }
            }
            __syncthreads();
            {   // o[j][d] = sum_t p[j][t] v[t][d]: four position groups per (head, 4 dims), the
                // group partials then summed in group order
                const int nu = hg * (kPHD / 4);
                for (int idx = tid; idx < 4 * nu; idx += kPThreads) {
                    const int grp = idx / nu, u = idx % nu, j = u / (kPHD / 4), d4 = u % (kPHD / 4);
                    const float *pj = s_p + j * kPChunk;
                    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
                    for (int t = grp; t < i_nt; t += 4) {
                        const float pt = pj[t];
                        const float4 v = reinterpret_cast<const float4 *>(s_v + t * kPKRow)[d4];
                        o.x = fmaf(pt, v.x, o.x);
                        o.y = fmaf(pt, v.y, o.y);
                        o.z = fmaf(pt, v.z, o.z);
                        o.w = fmaf(pt, v.w, o.w);
                    }
                    reinterpret_cast<float4 *>(s_po)[grp * nu + u] = o;
                }
                __syncthreads();
                for (int idx = tid; idx < hg * kPHD; idx += kPThreads) {
                    const int j = idx / kPHD, d = idx % kPHD, u4 = j * kPHD + d;
                    const float o = ((s_po[u4] + s_po[4 * nu + u4]) + s_po[8 * nu + u4]) + s_po[12 * nu + u4];
                    a.part[((size_t)(ig * hg + j) * a.nch_max + ich) * (kPHD + 2) + d] = o;
                }
            }
            mark(l, 4);
            if (l + 1 < a.L) release_and([&] { stage_kv(l + 1); });
        }
        if (!p_grid_sync(a, gen, &s_flag, slot + 1)) { drain(); return; }
        // ---------------- P3: merge, Wo rows, partial votes ----------------
        {
            constexpr int AR = (NV * 128 + kPThreads - 1) / kPThreads;  // att elements per thread
            float ov[AR][16];
#pragma unroll
            for (int r = 0; r < AR; r++) {
                const int i = tid + kPThreads * r;
#pragma unroll
                for (int c = 0; c < 16; c++) ov[r][c] = 0.f;
                if (i < D) {
                    const int h = i / kPHD, d = i % kPHD;
                    const float *pp = a.part + (size_t)h * a.nch_max * (kPHD + 2) + d;
#pragma unroll
                    for (int c = 0; c < 16; c++)
                        if (c < nch) ov[r][c] = __ldcg(pp + (size_t)c * (kPHD + 2));
                }
            }
            for (int idx = tid; idx < a.H * nch; idx += kPThreads) {
                const int h = idx / nch, c = idx % nch;
                const float *pp = a.part + ((size_t)h * a.nch_max + c) * (kPHD + 2) + kPHD;
                s_ml[2 * (h * a.nch_max + c)] = __ldcg(pp);
                s_ml[2 * (h * a.nch_max + c) + 1] = __ldcg(pp + 1);
            }
            __syncthreads();
            if (tid < a.H) {
                const int h = tid;
                float M = -INFINITY;
                for (int c = 0; c < nch; c++) M = fmaxf(M, s_ml[2 * (h * a.nch_max + c)]);
                float S = 0.f;
                for (int c = 0; c < nch; c++) {
                    const float f = expf(s_ml[2 * (h * a.nch_max + c)] - M);
                    s_fm[h * a.nch_max + c] = f;
                    S = fmaf(s_ml[2 * (h * a.nch_max + c) + 1], f, S);
                }
                for (int c = 0; c < nch; c++) s_fm[h * a.nch_max + c] = s_fm[h * a.nch_max + c] / S;
            }
            __syncthreads();
#pragma unroll
            for (int r = 0; r < AR; r++) {
                const int i = tid + kPThreads * r;
                if (i < D) {
                    const int h = i / kPHD;
                    float o = 0.f;
#pragma unroll
                    for (int c = 0; c < 16; c++)
                        if (c < nch) o = fmaf(ov[r][c], s_fm[h * a.nch_max + c], o);
                    s_att[i] = o;
                }
            }
            __syncthreads();
            mark(l, 5);
            wait_bar(2);
            for (int rr = warp; rr < nr; rr += kPWarps) {
                const float *wr = s_wo + (size_t)rr * D;
                float acc = 0.f;
#pragma unroll
                for (int j = 0; j < NV; j++) {
                    const int i4 = lane + 32 * j;
                    acc = dot4(reinterpret_cast<const float4 *>(wr)[i4], reinterpret_cast<const float4 *>(s_att)[i4], acc);
                }
                acc = warp_sum(acc);
                if (lane == 0) {
                    const float xn = __fadd_rn(s_xr[rr], acc);
                    s_xr[rr] = xn;
                    a.x[d0 + rr] = xn;
                }
            }
            __syncthreads();
            if (tid < 16) {
                float pv = 0.f;
                for (int rr = 0; rr < nr; rr++) pv = __fadd_rn(pv, __fmul_rn(wvn[rr * 16 + tid], s_xr[rr]));
                a.vpart[(size_t)blockIdx.x * 17 + tid] = pv;
            } else if (tid == 16) {
                float ss = 0.f;
                for (int rr = 0; rr < nr; rr++) ss = __fadd_rn(ss, __fmul_rn(s_xr[rr], s_xr[rr]));
                a.vpart[(size_t)blockIdx.x * 17 + 16] = ss;
            }
            if (l + 1 < a.L) release_and([&] { stage_wo(l + 1); });
        }
        if (!p_grid_sync(a, gen, &s_flag, slot + 2)) { drain(); return; }
        // ---------------- P4: election + gate/up of the elected experts ----------------
        {
            if (warp < 5) {  // totals in a fixed order: 8 strided partial sums per slot, then a tree
                const int q = tid >> 3, s8 = tid & 7;
                float vals[256 / 8];
#pragma unroll
                for (int j = 0; j < 256 / 8; j++) {
                    const int c = s8 + 8 * j;
                    vals[j] = (q < 17 && c < G) ? __ldcg(a.vpart + (size_t)c * 17 + q) : 0.f;
                }
                float acc = 0.f;
#pragma unroll
                for (int j = 0; j < 256 / 8; j++)
                    if (s8 + 8 * j < G) acc = __fadd_rn(acc, vals[j]);
#pragma unroll
                for (int o = 4; o; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(JDG_FULL, acc, o, 8));
                if (s8 == 0 && q < 17) tot[q] = acc;
            }
            // the FFN input x after attention (all model rows)
            p_g2s<4>(reinterpret_cast<float4 *>(s_x), reinterpret_cast<const float4 *>(a.x), D / 4);
            __syncthreads();
            if (warp == 0) p_elect_warp0(tot, ly.alive, ema_s[l], ly.temperature, D, a.eps, eo);
            __syncthreads();
            mark(l, 6);
            const int k = eo.k;
            if (blockIdx.x == 0 && tid < kMaxE) {
                a.tr_sel[(size_t)l * kMaxE + tid] = eo.sel[tid];
                a.tr_w[(size_t)l * kMaxE + tid] = eo.w[tid];
                if (tid == 0) {
                    a.tr_k[l] = k;
                    a.tr_ema[l] = eo.ema;
                    a.consensus[l] = eo.ema;
                    atomicAdd(a.stats, (unsigned long long)k);
                }
            }
            const float inv = eo.inv;
            for (int i = tid; i < D; i += kPThreads) s_x[i] = __fmul_rn(__fmul_rn(s_x[i], inv), ffn_norm[i]);
            // the down rows this CTA reads in P5, into L2 while the gate/up rows stream
            if (tid < k * nr) {
                const int ki = tid / nr, rr = tid % nr;
                p_prefetch_range(ly.dn[eo.sel[ki]] + (size_t)(d0 + rr) * a.hidden, (size_t)a.hidden * 4);
            }
            if (tid < kMaxE) s_gub[tid] = tid < k ? ly.gu[eo.sel[tid]] : nullptr;
            __syncthreads();
            const float *const *gub = s_gub;
            const int nunits = k * a.hidden, gw = G * kPWarps;
            float4 ga[NV], ua[NV], gb[NV], ub[NV];
            auto load_unit = [&](int uu, float4(&g4)[NV], float4(&u4)[NV]) {
                if (uu >= nunits) return;
                const int ki = uu / a.hidden, i = uu - ki * a.hidden;
                const float *g = gub[ki] + (size_t)(2 * i) * D, *up = g + D;
#pragma unroll
                for (int j = 0; j < NV; j++) {
                    g4[j] = ld_stream4(g + 4 * (lane + 32 * j));
                    u4[j] = ld_stream4(up + 4 * (lane + 32 * j));
                }
            };
            auto compute_unit = [&](int uu, const float4(&g4)[NV], const float4(&u4)[NV]) {
                float ag = 0.f, au = 0.f;
#pragma unroll
                for (int j = 0; j < NV; j++) {
                    const float4 xv = reinterpret_cast<const float4 *>(s_x)[lane + 32 * j];
                    ag = dot4(g4[j], xv, ag);
                    au = dot4(u4[j], xv, au);
                }
                ag = warp_sum(ag);
                au = warp_sum(au);
                if (lane == 0) a.hbuf[uu] = __fmul_rn(silu_ref(ag), au);
            };
            int u = blockIdx.x * kPWarps + warp;
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
        if (!p_grid_sync(a, gen, &s_flag, slot + 3)) { drain(); return; }
        // ---------------- P5: down rows of the elected experts, combined into x ----------------
        {
            const int k = eo.k;
            p_g2s<8>(reinterpret_cast<float4 *>(s_h), reinterpret_cast<const float4 *>(a.hbuf), k * a.hidden / 4);
            __syncthreads();
            mark(l, 7);
            // pairs (row rr, election slot ki) per warp, two in flight
            const int np = nr * k;
            float4 wa[NH], wb[NH];
            auto load_pair = [&](int pr, float4(&w4)[NH]) {
                if (pr >= np) return;
                const int rr = pr / k, ki = pr % k;
                const float *w = ly.dn[eo.sel[ki]] + (size_t)(d0 + rr) * a.hidden;
#pragma unroll
                for (int j = 0; j < NH; j++) w4[j] = ld_stream4(w + 4 * (lane + 32 * j));
            };
            auto compute_pair = [&](int pr, const float4(&w4)[NH]) {
                const int rr = pr / k, ki = pr % k;
                const float4 *h4 = reinterpret_cast<const float4 *>(s_h + (size_t)ki * a.hidden);
                float acc = 0.f;
#pragma unroll
                for (int j = 0; j < NH; j++) acc = dot4(w4[j], h4[lane + 32 * j], acc);
                acc = warp_sum(acc);
                if (lane == 0) s_y[rr * kMaxE + ki] = acc;
            };
            int pr = warp;
            load_pair(pr, wa);
            while (pr < np) {
                load_pair(pr + kPWarps, wb);
                compute_pair(pr, wa);
                pr += kPWarps;
                if (pr >= np) break;
                load_pair(pr + kPWarps, wa);
                compute_pair(pr, wb);
                pr += kPWarps;
            }
            __syncthreads();
            if (tid < nr) {
                float e = 0.f;
                for (int ki = 0; ki < k; ki++) e = __fadd_rn(e, __fmul_rn(eo.w[ki], s_y[tid * kMaxE + ki]));
                a.x[d0 + tid] = __fadd_rn(s_xr[tid], e);
            }
            fence_proxy_async_smem();  // s_par[l & 1] is refilled (layer l + 2) after the barrier
        }
        if (!p_grid_sync(a, gen, &s_flag, slot + 4)) { drain(); return; }
    }
    // ---------------- LM head: final RMSNorm, logits, greedy pick ----------------
    const int lslot = 1 + 5 * a.L;
    if (!misc_ready) wait_bar(5);
    p_g2s<4>(reinterpret_cast<float4 *>(s_x), reinterpret_cast<const float4 *>(a.x), D / 4);
    __syncthreads();
    float ss = 0.f;
    for (int i = tid; i < D / 4; i += kPThreads) {
        const float4 v = reinterpret_cast<const float4 *>(s_x)[i];
        ss = dot4(v, v, ss);
    }
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)D + a.eps);
    for (int i = tid; i < D; i += kPThreads) s_x[i] = __fmul_rn(__fmul_rn(s_x[i], inv), s_onorm[i]);
    __syncthreads();
    float val = -INFINITY;
    int vi = 0x7fffffff;
    {
        const int gw = G * kPWarps, npair = (a.V + 1) / 2;
        float4 wa[2][NV], wb[2][NV];
        auto load_pair = [&](int pr, float4(&w4)[2][NV]) {
            if (pr >= npair) return;
#pragma unroll
            for (int r = 0; r < 2; r++) {
                const int row = 2 * pr + r;
                if (row < a.V) {
                    const float *wr = a.output + (size_t)row * D;
#pragma unroll
                    for (int j = 0; j < NV; j++) w4[r][j] = ld_stream4(wr + 4 * (lane + 32 * j));
                }
            }
        };
        auto compute_pair = [&](int p2, const float4(&w4)[2][NV]) {
            float acc[2] = {0.f, 0.f};
#pragma unroll
            for (int j = 0; j < NV; j++) {
                const float4 xv = reinterpret_cast<const float4 *>(s_x)[lane + 32 * j];
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
        int pr = blockIdx.x * kPWarps + warp;
        load_pair(pr, wa);
        while (pr < npair) {
            load_pair(pr + gw, wb);
            compute_pair(pr, wa);
            pr += gw;
            if (pr >= npair) break;
            load_pair(pr + gw, wa);
            compute_pair(pr, wb);
            pr += gw;
        }
    }
    if (lane == 0) {
        bv_s[warp] = val;
        bi_s[warp] = vi;
    }
    __syncthreads();
    if (tid == 0) {
        float bv = bv_s[0];
        int bi = bi_s[0];
        for (int q = 1; q < kPWarps; q++)
            if (bv_s[q] > bv || (bv_s[q] == bv && bi_s[q] < bi)) {
                bv = bv_s[q];
                bi = bi_s[q];
            }
        a.amax_v[blockIdx.x] = bv;
        a.amax_i[blockIdx.x] = bi;
    }
    if (a.tl && tid == 0) atomicMax(a.tl + 3 * lslot + 2, p_gtimer());
    if (!a.greedy_pick) return;
    // the last CTA to finish takes the first-index maximum (janusdoe.c:3637) or the prompt's
    // next id and advances tok / pos / history
    __shared__ unsigned s_ticket;
    __threadfence();
    __syncthreads();
    if (tid == 0) s_ticket = atomicAdd(a.ticket, 1u);
    __syncthreads();
    if (s_ticket != (unsigned)G - 1) return;
    __threadfence();
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int q = tid; q < G; q += kPThreads) {
        const float v = __ldcg(a.amax_v + q);
        const int i = __ldcg(a.amax_i + q);
        if (v > bv || (v == bv && i < bi)) {
            bv = v;
            bi = i;
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
    if (tid == 0) {
        for (int q = 1; q < kPWarps; q++)
            if (bv_s[q] > bv_s[0] || (bv_s[q] == bv_s[0] && bi_s[q] < bi_s[0])) {
                bv_s[0] = bv_s[q];
                bi_s[0] = bi_s[q];
            }
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
        *a.ticket = 0;
    }
}

}  // namespace jdg

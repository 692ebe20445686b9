// jdg_tc32.cuh — f32-accurate GEMM on the tcgen05 tensor cores for the own model's batched
// step (q/k/v, Wo, the elected experts' gate/up and down, the LM head):
//
//     C[t][n] = sum_k X[t][k] * W[n][k]      (t: token rows, n: weight rows)
//
// The f32 operands are split into TF32 parts, x = x_hi + x_lo with x_hi = x rounded to 10
// mantissa bits and x_lo = x - x_hi (exact in f32, |x_lo| <= 2^-11 |x|; the tensor core keeps
// its top 10 bits, so 2^-22 |x|), and three kind::tf32 products are accumulated in f32 in
// tensor memory: W_hi.X_hi + W_hi.X_lo + W_lo.X_hi.  Every product of two TF32 numbers is
// exact in f32; the omitted W_lo.X_lo is at most 2^-22 |w x| per term (about 2^-24 on
// average), which over a K = 768 sum stays an order of magnitude below the rounding of the
// f32 sum itself (measured on N(0, 0.02) weights: 7.5e-8 against 4.3e-7 relative).
//
// Operands live in global memory already in the shared-memory layout the MMA descriptors
// address (canonical K-major, no swizzle): for a block of 128 rows and a 32-wide K chunk, the
// core matrix (row group g < 16, K group c < 8) of 8 rows x 4 elements (16 bytes a row) sits
// at byte (c * 16 + g) * 128 — 16 KB per block and part.  Weights are laid out once at upload
// ([row tile][K chunk][hi | lo]); activations by a prep kernel before each product
// ([segment][token tile][K chunk][hi | lo], rows past the segment's count left as they are).  So a stage
// is four 1-D bulk copies (cp.async.bulk, no tensor maps), and every byte is read once.
//
// CTA (352 threads) = one 128-row x 128-token output tile over a K range (split-K CTAs write
// partials that k_tc_reduce adds in split order): thread 0 streams stages into a 3-deep ring;
// threads 32 and 320 issue (alternate chunks) the 12 MMAs (M128 K8, N = the tile's token count rounded up to 32) of each
// 32-wide chunk into one of four accumulator regions and commits the stage back; warps 2-9 drain each
// chunk's region into f32 registers with round-to-nearest adds (the tensor core's own
// accumulation then spans only one chunk, 128 products) and apply the epilogue.  Every wait is bounded by wall time; on a timeout the CTA flags
// JDG_ERR_TIMEOUT, waits (bounded) for what it issued, frees its tensor memory and returns.
#pragma once
#include "jdg_async.cuh"
#include "jdg_kernels.cuh"

namespace jdg {

constexpr int kTcRows = 128;                   // weight rows per tile (MMA M)
constexpr int kTcTok = 128;                    // tokens per tile (MMA N)
constexpr int kTcK = 32;                       // K elements per chunk (one stage)
constexpr int kTcBlk = kTcRows * kTcK * 4;     // 16 KB: one part of one operand block
constexpr int kTcStages = 3;
constexpr int kTcStageBytes = 4 * kTcBlk;      // W hi, W lo, X hi, X lo
constexpr int kTcSmem = 1024 + kTcStages * kTcStageBytes;
constexpr int kTcMaxSplit = 8;
constexpr int kTcThreads = 352;                // warp 0 copies, warps 1 and 10 MMAs, warps 2-9 drain
constexpr int kTcDrainCols = 64;               // token columns per drain warp (two warps per TMEM lane quarter)
static_assert(kTcTok == kSplitTile && kTcRows == kSplitTile && kTcMaxSplit <= kSplitMax, "split_sum reads the partial tiles");
constexpr int kTcRegions = 4;                  // accumulator regions of 128 TMEM columns
// kind::tf32 instruction descriptor: D f32 (bits 4-5 = 1), A and B TF32 (bits 7-9, 10-12 = 2),
// both K-major, M = 128 (bits 24-28 = M/16); N (bits 17-22 = N/8) is set per tile
constexpr uint32_t kTcIdescM = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(kTcRows >> 4) << 24);
__host__ __device__ __forceinline__ uint32_t tc_idesc(int n) { return kTcIdescM | ((uint32_t)(n >> 3) << 17); }

// byte offset of element (row r, k) inside a 128 x 32 block
__host__ __device__ __forceinline__ uint32_t tc_off(int r, int k) {
    return (uint32_t)((((k >> 2) * 16 + (r >> 3)) * 128) + (r & 7) * 16 + (k & 3) * 4);
}
// x = hi + lo: hi is x rounded to 10 mantissa bits (ties away from zero), lo = x - hi is exact
// in f32 with |lo| <= 2^-11 |x|, and the tensor core's TF32 view of lo keeps it to 2^-22 |x|
__device__ __forceinline__ void tc_split(float x, float &hi, float &lo) {
    hi = __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
    lo = x - hi;
}

// Weight blocks of an N x K f32 matrix (rows past N zero): grid-stride over (row, 4-element group).
static __global__ void k_tc_wprep(const float *__restrict__ W, int N, int K, uint8_t *__restrict__ out) {
    const int nkc = K / kTcK, rt_n = (N + kTcRows - 1) / kTcRows;
    const long total = (long)rt_n * kTcRows * (K / 4);
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int row = (int)(i / (K / 4)), k4 = (int)(i % (K / 4)) * 4;
        const int rt = row / kTcRows, r = row % kTcRows, kc = k4 / kTcK, k = k4 % kTcK;
        float4 v = row < N ? *reinterpret_cast<const float4 *>(W + (size_t)row * K + k4) : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 h, l;
        tc_split(v.x, h.x, l.x);
        tc_split(v.y, h.y, l.y);
        tc_split(v.z, h.z, l.z);
        tc_split(v.w, h.w, l.w);
        uint8_t *blk = out + ((size_t)rt * nkc + kc) * 2 * kTcBlk;
        *reinterpret_cast<float4 *>(blk + tc_off(r, k)) = h;
        *reinterpret_cast<float4 *>(blk + kTcBlk + tc_off(r, k)) = l;
    }
}

// Activation blocks: segment s, token j of the segment is row idx[s*ldi + j] of X (idx null:
// row j, segment 0), j < cnt[s] (cnt null: M).  Rows past the count are not written: they
// only reach output columns (tokens) that are never stored.
// out: [seg][token tile < ttiles][K chunk][hi | lo][16 KB]
struct TcPrep {
    const float *X;
    long x_seg;  // row base of segment s: X + s * x_seg
    int ldx, K;
    const int *idx;
    int ldi;
    const int *cnt;
    int M, nseg, ttiles;
    int glu;  // 1: X rows hold interleaved (gate, up) pairs, 2K floats; the product reads silu(gate) * up
    uint8_t *out;
};
static __global__ void k_tc_xprep(TcPrep p) {
    const int nkc = p.K / kTcK;
    // 32-bit index arithmetic: the engine uses this path only when 16 segments x (rows + 128)
    // x K/4 stays below 2^32
    const unsigned kq = (unsigned)p.K / 4, per_seg = (unsigned)p.ttiles * kTcTok * kq;
    const unsigned total = per_seg * (unsigned)p.nseg;
    for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const unsigned s = i / per_seg, rem = i - s * per_seg;
        const int j = (int)(rem / kq), k4 = (int)(rem - (unsigned)j * kq) * 4;
        const int n = p.cnt ? p.cnt[s] : p.M;
        if (j >= n) continue;
        const int row = p.idx ? p.idx[(size_t)s * p.ldi + j] : j;
        float4 v;
        if (p.glu) {  // janusdoe.c:925: silu(gate) * up, in f32
            const float *xr = p.X + (size_t)s * p.x_seg + (size_t)row * p.ldx + 2 * k4;
            const float4 a = *reinterpret_cast<const float4 *>(xr), b = *reinterpret_cast<const float4 *>(xr + 4);
            v = make_float4(__fmul_rn(silu_ref(a.x), a.y), __fmul_rn(silu_ref(a.z), a.w), __fmul_rn(silu_ref(b.x), b.y),
                            __fmul_rn(silu_ref(b.z), b.w));
        } else {
            v = *reinterpret_cast<const float4 *>(p.X + (size_t)s * p.x_seg + (size_t)row * p.ldx + k4);
        }
        float4 h, l;
        tc_split(v.x, h.x, l.x);
        tc_split(v.y, h.y, l.y);
        tc_split(v.z, h.z, l.z);
        tc_split(v.w, h.w, l.w);
        const int tt = j / kTcTok, t = j % kTcTok, kc = k4 / kTcK, k = k4 % kTcK;
        uint8_t *blk = p.out + (((size_t)s * p.ttiles + tt) * nkc + kc) * 2 * kTcBlk;
        *reinterpret_cast<float4 *>(blk + tc_off(t, k)) = h;
        *reinterpret_cast<float4 *>(blk + kTcBlk + tc_off(t, k)) = l;
    }
}

// Activation blocks written by the kernel that produces the activations (no separate prep):
// one f32 value v of row j, column k of a single-segment operand with ttiles token tiles.
__device__ __forceinline__ void tc_put(uint8_t *__restrict__ out, int nkc, int j, int k, float v) {
    float hi, lo;
    tc_split(v, hi, lo);
    uint8_t *blk = out + ((size_t)(j / kTcTok) * nkc + k / kTcK) * 2 * kTcBlk;
    *reinterpret_cast<float *>(blk + tc_off(j % kTcTok, k % kTcK)) = hi;
    *reinterpret_cast<float *>(blk + kTcBlk + tc_off(j % kTcTok, k % kTcK)) = lo;
}

// RMS norm of row b (janusdoe.c:504, the arithmetic of k_rmsnorm) written straight into the
// activation blocks of the next product.  grid = rows, block 256.
static __global__ void k_tc_norm_prep(const float *__restrict__ x, const float *__restrict__ w, int D, float eps,
                                      uint8_t *__restrict__ out) {
    __shared__ float red[32];
    const int b = blockIdx.x, nkc = D / kTcK;
    const float *xr = x + (size_t)b * D;
    const float inv = rms_inv(xr, D, eps, red);
    for (int k4 = threadIdx.x * 4; k4 < D; k4 += blockDim.x * 4) {
        const float4 v = *reinterpret_cast<const float4 *>(xr + k4), g = *reinterpret_cast<const float4 *>(w + k4);
        float4 y = make_float4(__fmul_rn(__fmul_rn(v.x, inv), g.x), __fmul_rn(__fmul_rn(v.y, inv), g.y),
                               __fmul_rn(__fmul_rn(v.z, inv), g.z), __fmul_rn(__fmul_rn(v.w, inv), g.w));
        float4 h, l;
        tc_split(y.x, h.x, l.x);
        tc_split(y.y, h.y, l.y);
        tc_split(y.z, h.z, l.z);
        tc_split(y.w, h.w, l.w);
        uint8_t *blk = out + ((size_t)(b / kTcTok) * nkc + k4 / kTcK) * 2 * kTcBlk;
        *reinterpret_cast<float4 *>(blk + tc_off(b % kTcTok, k4 % kTcK)) = h;
        *reinterpret_cast<float4 *>(blk + kTcBlk + tc_off(b % kTcTok, k4 % kTcK)) = l;
    }
}

// Attention merge (k_attn_combine's arithmetic) written into the activation blocks of the Wo
// product: grid (H, rows), block HD, dynamic shared memory 2 * nchunk floats.
static __global__ void k_tc_combine_prep(const float *__restrict__ part, const int *__restrict__ pos, int H, int HD,
                                         int nchunk, int chunk, uint8_t *__restrict__ out) {
    extern __shared__ float tcp_ml[];
    const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    const int nc = pos[b] / chunk + 1;
    const float o = attn_merge(part + ((size_t)b * H + h) * nchunk * (HD + 2), nc, HD, d, tcp_ml);
    tc_put(out, H * HD / kTcK, b, h * HD + d, o);
}

struct TcArgs {
    const uint8_t *const *wt;  // per segment: weight blocks of W (n_rows x K); null = no work
    const uint8_t *xt;         // activation blocks [seg][ttiles][nkc][2][16 KB]
    const int *cnt;            // per segment token counts (null: M, one segment)
    int M, n_rows, nkc, ttiles;
    float *C;                  // C[seg * c_seg + t * ldc + col]
    int ldc;
    long c_seg;
    int epi;                   // EPI_STORE, EPI_ADD (C += alpha * Y), EPI_SWIGLU (C[t][n/2] = silu(Y[2i]) * Y[2i+1])
    float alpha;
    int ksplit;
    float *part;               // [tiles][ksplit][128 tokens][128 rows], tile = (seg * ttiles + tt) * rtiles + rt
    int *err;
    unsigned long long *tl;    // optional wait profile (engine debug timeline), null when off
    int tl_type;               // product kind: its eight counters are timeline slots 400 + 8 * tl_type
};

__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr) {
    // LBO (K-direction core-matrix stride) = 16 row groups x 128 B, SBO (row-group stride) = 128
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((2048u >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((128u >> 4) & 0x3FFF) << 32) | (1ull << 46);
}
__device__ __forceinline__ void tc_mma(uint32_t dtmem, uint64_t da, uint64_t db, uint32_t acc, uint32_t idesc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %3, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %4, p; }" ::"r"(dtmem),
        "l"(da), "l"(db), "r"(acc), "r"(idesc));
}
__device__ __forceinline__ unsigned long long tc_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// mbarrier phase wait bounded by 200 ms of wall time
__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity) {
    const unsigned long long t0 = tc_now();
    for (int it = 0;; it++) {
        uint32_t done;
        asm volatile("{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                     : "=r"(done)
                     : "r"(smem_u32(bar)), "r"(parity)
                     : "memory");
        if (done) return true;
        if ((it & 63) == 63 && tc_now() - t0 > 200ull * 1000 * 1000) return false;
    }
}

// The same wait for threads with nothing else to do (copy thread, drain warps): after one
// test, mbarrier.try_wait suspends the thread in hardware until the phase completes or a
// short time passes, so the waiters do not take issue slots from the MMA thread.
__device__ __forceinline__ bool tc_wait_idle(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile("{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(done)
                 : "r"(smem_u32(bar)), "r"(parity)
                 : "memory");
    if (done) return true;
    const unsigned long long t0 = tc_now();
    for (;;) {
        asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                     : "=r"(done)
                     : "r"(smem_u32(bar)), "r"(parity)
                     : "memory");
        if (done) return true;
        if (tc_now() - t0 > 200ull * 1000 * 1000) return false;
    }
}
// 8 consecutive f32 columns (tokens) of this warp's 32 TMEM lanes (rows), waited for
__device__ __forceinline__ void tc_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}

// the same without the wait (several loads in flight, then one tcgen05.wait::ld)
__device__ __forceinline__ void tc_ld8_nw(uint32_t taddr, float *v) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tc_store(const TcArgs &a, int seg, int t, int n, float v, int lane) {
    float *c = a.C + (size_t)seg * a.c_seg + (size_t)t * a.ldc;
    if (a.epi == EPI_SWIGLU) {
        const float other = __shfl_xor_sync(JDG_FULL, v, 1);  // every lane takes part
        if ((lane & 1) == 0 && n + 1 < a.n_rows) c[n >> 1] = __fmul_rn(silu_ref(v), other);
    } else if (n < a.n_rows) {
        if (a.epi == EPI_ADD) c[n] = __fadd_rn(c[n], __fmul_rn(v, a.alpha));
        else c[n] = v;
    }
}

static __global__ __launch_bounds__(kTcThreads, 1) void k_tc32_gemm(TcArgs a) {
    extern __shared__ __align__(1024) uint8_t tc_sm[];
    uint8_t *stages = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tc_sm) + 1023) & ~(uintptr_t)1023);
    __shared__ __align__(8) uint64_t full[kTcStages], empty[kTcStages], ready[kTcRegions], freed[kTcRegions];
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    __shared__ int seen[2];  // chunks of each parity whose operands their MMA issuer has seen land
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rt = blockIdx.x, tt = blockIdx.y, seg = blockIdx.z / a.ksplit, ks = blockIdx.z % a.ksplit;
    const int n_tok_seg = a.cnt ? a.cnt[seg] : a.M;
    const int ntok = min(kTcTok, n_tok_seg - tt * kTcTok);
    const uint8_t *wt = a.wt[seg];
    if (ntok <= 0 || !wt) return;  // whole CTA, before any barrier or allocation
    const bool prof = a.tl != nullptr;
    long long pw = 0, pw2 = 0;
    const long long t_begin = prof ? clock64() : 0;
    const int per = (a.nkc + a.ksplit - 1) / a.ksplit, kc0 = ks * per, kc1 = min(a.nkc, kc0 + per);
    const int nloc = max(0, kc1 - kc0);
    if (tid == 0) {
        for (int s = 0; s < kTcStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int q = 0; q < kTcRegions; q++) {
            mbar_init(&ready[q], 1);
            mbar_init(&freed[q], 8);  // the eight drain warps
        }
        abort_flag = 0;
        seen[0] = seen[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(kTcRegions * kTcTok));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_slot;
    // debug wait profile (clock64 cycles): [1] CTA, [2] copy waits, [3] MMA operand waits,
    // [4] MMA region waits, [5] drain waits (warp 2), [6] drain epilogue, [7] set-up
    if (prof && tid == 0) {
        unsigned long long *c = a.tl + 3 * (400 + 8 * a.tl_type) + 2;
        atomicAdd(c, 1ull);
        atomicAdd(c + 3 * 7, (unsigned long long)(clock64() - t_begin));
    }
    const uint8_t *wbase = wt + ((size_t)rt * a.nkc) * 2 * kTcBlk;
    const uint8_t *xbase = a.xt + (((size_t)seg * a.ttiles + tt) * a.nkc) * 2 * kTcBlk;
    int issued_ld = 0, issued_mma = 0;
    if (tid == 0) {
        // ---------------- producer: four 16 KB bulk copies per chunk ----------------
        for (int i = 0; i < nloc; i++) {
            const int s = i % kTcStages;
            const long long w0 = prof ? clock64() : 0;
            if (i >= kTcStages && !tc_wait_idle(&empty[s], (uint32_t)((i / kTcStages) - 1) & 1u)) {
                abort_flag = 1;
                break;
            }
            if (prof) pw += clock64() - w0;
            if (*(volatile int *)&abort_flag) break;
            uint8_t *st = stages + (size_t)s * kTcStageBytes;
            const int kc = kc0 + i;
            mbar_expect_tx(&full[s], kTcStageBytes);
            bulk_g2s(st, wbase + (size_t)kc * 2 * kTcBlk, 2 * kTcBlk, &full[s]);
            bulk_g2s(st + 2 * kTcBlk, xbase + (size_t)kc * 2 * kTcBlk, 2 * kTcBlk, &full[s]);
            issued_ld = i + 1;
        }
    } else if (tid == 32 || tid == kTcThreads - 32) {
        // ---------------- MMA issuers: chunk i into accumulator region i % kTcRegions ----------------
        // thread 32 issues the even chunks, the first thread of warp 10 the odd ones (each
        // commit tracks the issuing thread's own MMAs; different chunks use different stages
        // and regions), so one chunk's issue overlaps the other's waits
        // token columns past ntok are not computed beyond the next multiple of 32; the drain
        // reads whole groups of 32 columns and stores only those below ntok
        const uint32_t idesc = tc_idesc(min(kTcTok, (ntok + 31) & ~31));
        const int par = tid == 32 ? 0 : 1;
        for (int i = par; i < nloc; i += 2) {
            const int s = i % kTcStages, q = i % kTcRegions;
            const long long w0 = prof ? clock64() : 0;
            bool ok = true;
            if (i >= kTcStages) {
                // stage s last held chunk i - 3, the other issuer's: its phase of full[s] must
                // have completed before this parity test means chunk i (a phase-parity wait
                // cannot tell phase n from phase n - 2)
                const int o = (i - kTcStages) & 1, need = (i - kTcStages - o) / 2 + 1;
                const unsigned long long t0 = tc_now();
                while (*(volatile int *)&seen[o] < need)
                    if (tc_now() - t0 > 200ull * 1000 * 1000) {
                        ok = false;
                        break;
                    }
            }
            ok = ok && tc_wait(&full[s], (uint32_t)(i / kTcStages) & 1u);
            if (ok) *(volatile int *)&seen[par] = (i - par) / 2 + 1;
            const long long w1 = prof ? clock64() : 0;
            if (ok && i >= kTcRegions) ok = tc_wait(&freed[q], (uint32_t)((i / kTcRegions) - 1) & 1u);
            if (prof) {
                pw += w1 - w0;
                pw2 += clock64() - w1;
            }
            if (!ok || *(volatile int *)&abort_flag) {
                abort_flag = 1;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t st = smem_u32(stages + (size_t)s * kTcStageBytes);
            // descriptors of the four parts; a K slice moves the start address (bits 0-13,
            // 16-byte units) by two K groups of 2048 bytes
            const uint64_t dwh = tc_desc(st), dwl = tc_desc(st + kTcBlk), dxh = tc_desc(st + 2 * kTcBlk),
                           dxl = tc_desc(st + 3 * kTcBlk);
            const uint32_t d = tmem + (uint32_t)(q * kTcTok);
#pragma unroll
            for (int k8 = 0; k8 < kTcK / 8; k8++) {  // K slices of 8: two K groups of the block
                const uint64_t o = (uint64_t)(k8 * 2 * 2048 >> 4);
                tc_mma(d, dwh + o, dxh + o, k8 > 0 ? 1u : 0u, idesc);
                tc_mma(d, dwh + o, dxl + o, 1u, idesc);
                tc_mma(d, dwl + o, dxh + o, 1u, idesc);
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_u32(&empty[s]))
                         : "memory");
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_u32(&ready[q]))
                         : "memory");
            issued_mma = i + 1;
        }
    }
    __syncwarp();
    if (warp >= 2 && warp < 10) {
        // ---------------- drain: every chunk's product added in f32 (round to nearest) ----------------
        // warp w reads TMEM lanes 32 (w % 4) .. (its weight rows), token columns
        // col0 .. col0 + 63: all eight 8-column loads in flight before one wait
        const int quarter = warp & 3, row = quarter * 32 + lane, n = rt * kTcRows + row;
        const int col0 = ((warp - 2) >> 2) * kTcDrainCols, ncol = min(kTcDrainCols, ntok - col0);
        float acc[kTcDrainCols];
#pragma unroll
        for (int c = 0; c < kTcDrainCols; c++) acc[c] = 0.f;
        bool ok = true;
        for (int i = 0; i < nloc; i++) {
            const int q = i % kTcRegions;
            const long long w0 = prof ? clock64() : 0;
            if (!tc_wait_idle(&ready[q], (uint32_t)(i / kTcRegions) & 1u)) ok = false;
            if (prof) pw += clock64() - w0;
            if (__any_sync(JDG_FULL, !ok || *(volatile int *)&abort_flag)) {  // leave as a whole warp
                ok = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t base = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(q * kTcTok + col0);
            if (ncol > 32) {  // uniform per warp; columns past ntok (up to the MMA's N) are not stored
                float v[64];
#pragma unroll
                for (int j = 0; j < 64; j += 8) tc_ld8_nw(base + (uint32_t)j, v + j);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int j = 0; j < 64; j++) acc[j] = __fadd_rn(acc[j], v[j]);
            } else if (ncol > 0) {
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; j += 8) tc_ld8_nw(base + (uint32_t)j, v + j);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int j = 0; j < 32; j++) acc[j] = __fadd_rn(acc[j], v[j]);
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&freed[q]);
        }
        if (!ok) abort_flag = 1;
        const long long e0 = prof ? clock64() : 0;
        // Epilogue.  The tile goes through shared memory (the stage ring is idle once every
        // chunk's product has been drained) as [token][row] and leaves by bulk copies, one row
        // of the output per token; a residual add, or rows/strides that are not 16-byte
        // multiples, take per-thread stores instead.
        const int nr = min(kTcRows, a.n_rows - rt * kTcRows);
        const bool al16 = a.ldc % 4 == 0 && a.c_seg % 4 == 0 && (reinterpret_cast<uintptr_t>(a.C) & 15) == 0;
        const bool bulk = a.ksplit > 1 || (a.epi == EPI_STORE && al16 && nr % 4 == 0) ||
                          (a.epi == EPI_SWIGLU && al16 && nr % 8 == 0);
        if (!bulk) {
            if (ok && nloc > 0) {
#pragma unroll
                for (int c = 0; c < kTcDrainCols; c++)
                    if (c < ncol) tc_store(a, seg, tt * kTcTok + col0 + c, n, acc[c], lane);
            }
        } else {
            float *tile = reinterpret_cast<float *>(stages);  // [128 tokens][128 rows]
            if (ok && nloc > 0) {  // this warp saw every chunk land: no copy into the ring is in flight
                if (a.ksplit == 1 && a.epi == EPI_SWIGLU) {
#pragma unroll
                    for (int c = 0; c < kTcDrainCols; c++)
                        if (c < ncol) {  // uniform per warp
                            const float other = __shfl_xor_sync(JDG_FULL, acc[c], 1);
                            if ((lane & 1) == 0) tile[(col0 + c) * kTcRows + (row >> 1)] = __fmul_rn(silu_ref(acc[c]), other);
                        }
                } else {
#pragma unroll
                    for (int c = 0; c < kTcDrainCols; c++)
                        if (c < ncol) tile[(col0 + c) * kTcRows + row] = acc[c];
                }
            }
            fence_proxy_async_smem();
            asm volatile("bar.sync 1, 256;" ::: "memory");  // the eight drain warps
            if (lane == 0 && nloc > 0 && !*(volatile int *)&abort_flag) {
                if (a.ksplit > 1) {
                    if (warp == 2) {
                        const size_t t = ((size_t)seg * gridDim.y + tt) * gridDim.x + rt;
                        bulk_s2g(a.part + (t * a.ksplit + ks) * (size_t)kTcTok * kTcRows, tile,
                                 (uint32_t)ntok * kTcRows * 4);
                    }
                } else {
                    const bool glu = a.epi == EPI_SWIGLU;
                    float *cb = a.C + (size_t)seg * a.c_seg + (size_t)rt * (glu ? kTcRows / 2 : kTcRows);
                    for (int c = warp - 2; c < ntok; c += 8)
                        bulk_s2g(cb + (size_t)(tt * kTcTok + c) * a.ldc, tile + c * kTcRows, (uint32_t)(glu ? nr * 2 : nr * 4));
                }
                bulk_s2g_drain();
            }
        }
        if (prof && warp == 2 && lane == 0) {
            unsigned long long *c = a.tl + 3 * (400 + 8 * a.tl_type) + 2;
            atomicAdd(c + 3 * 5, (unsigned long long)pw);
            atomicAdd(c + 3 * 6, (unsigned long long)(clock64() - e0));
        }
    }
    __syncthreads();
    if (abort_flag) {
        if (tid == 0) atomicOr(a.err, JDG_ERR_TIMEOUT);
        // let the issued copies and MMAs land before the memory goes away
        if (tid == 0)
            for (int i = max(0, issued_ld - kTcStages); i < issued_ld; i++)
                tc_wait(&full[i % kTcStages], (uint32_t)(i / kTcStages) & 1u);
        if ((tid == 32 || tid == kTcThreads - 32) && issued_mma > 0) tc_wait(&empty[(issued_mma - 1) % kTcStages], (uint32_t)((issued_mma - 1) / kTcStages) & 1u);
    }
    if (prof && (tid == 0 || tid == 32 || tid == kTcThreads - 32)) {
        unsigned long long *c = a.tl + 3 * (400 + 8 * a.tl_type) + 2;
        if (tid == 0) atomicAdd(c + 3 * 2, (unsigned long long)pw);
        if (tid != 0) {
            atomicAdd(c + 3 * 3, (unsigned long long)pw);
            atomicAdd(c + 3 * 4, (unsigned long long)pw2);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (prof && tid == 0) atomicAdd(a.tl + 3 * (400 + 8 * a.tl_type) + 2 + 3, (unsigned long long)(clock64() - t_begin));
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcRegions * kTcTok));
    }
}

// Split-K sum: out[t][n] = sum over z = 0..ksplit-1 (in that order) of the partials, then the
// epilogue.  One thread per (tile, token, 4 consecutive rows), grid-stride.
static __global__ __launch_bounds__(256) void k_tc_reduce(TcArgs a, int rtiles, int nseg) {
    const long total = (long)nseg * a.ttiles * rtiles * kTcTok * (kTcRows / 4);
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int r4 = (int)(i % (kTcRows / 4)) * 4;
        const int c = (int)((i / (kTcRows / 4)) % kTcTok);
        const long tile = i / ((long)(kTcRows / 4) * kTcTok);
        const int rt = (int)(tile % rtiles), tt = (int)((tile / rtiles) % a.ttiles), seg = (int)(tile / ((long)rtiles * a.ttiles));
        const int n_tok_seg = a.cnt ? a.cnt[seg] : a.M;
        if (!a.wt[seg] || c >= n_tok_seg - tt * kTcTok) continue;
        const int n = rt * kTcRows + r4;
        if (n >= a.n_rows) continue;
        const float *p = a.part + (size_t)tile * a.ksplit * kTcTok * kTcRows + (size_t)c * kTcRows + r4;
        float4 pz[kTcMaxSplit];  // every split's partial loaded before the ordered sum
#pragma unroll
        for (int z = 0; z < kTcMaxSplit; z++)
            pz[z] = z < a.ksplit ? __ldcg(reinterpret_cast<const float4 *>(p + (size_t)z * kTcTok * kTcRows))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int z = 0; z < kTcMaxSplit; z++)
            if (z < a.ksplit) {
                s.x = __fadd_rn(s.x, pz[z].x);
                s.y = __fadd_rn(s.y, pz[z].y);
                s.z = __fadd_rn(s.z, pz[z].z);
                s.w = __fadd_rn(s.w, pz[z].w);
            }
        float *out = a.C + (size_t)seg * a.c_seg + (size_t)(tt * kTcTok + c) * a.ldc;
        const float v[4] = {s.x, s.y, s.z, s.w};
        if (a.epi == EPI_SWIGLU) {
#pragma unroll
            for (int j = 0; j < 4; j += 2)
                if (n + j + 1 < a.n_rows) out[(n + j) >> 1] = __fmul_rn(silu_ref(v[j]), v[j + 1]);
        } else {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                if (n + j >= a.n_rows) break;
                if (a.epi == EPI_ADD) out[n + j] = __fadd_rn(out[n + j], __fmul_rn(v[j], a.alpha));
                else out[n + j] = v[j];
            }
        }
    }
}

}  // namespace jdg

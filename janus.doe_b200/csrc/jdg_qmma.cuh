// jdg_qmma.cuh — batched host GEMM over Q4_K weights on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in tensor memory), for the host GGUF path at batch > 1.
//
//   Y[t][n] (epi)= sum_k X[t][k] * W[n][k],   W in Q4_K (janusdoe.c:2573-2585):
//   W[n][k] = d_sb * s_j * q - dmin_sb * m_j   (superblock sb of 256 weights, sub-block j of 32)
//
// Exact reformulation on fp16 tensor cores with f32 accumulation:
//   * A = s_j * q is an integer <= 63 * 15 = 945: exact in fp16.  The sub-block minimum
//     becomes a second product: A_min[n][j] = m_j (integer <= 63), against the sums of x over
//     each sub-block.
//   * X is split into x_hi = fp16(x) and x_lo = fp16(x - x_hi); together they carry ~22
//     mantissa bits.  B stacks them as 64 "columns": tokens 0..31 hi, then 0..31 lo.
//   * Per superblock one TMEM region receives A.B (K = 256, 16 MMAs of 128x64x16) and
//     A_min.B_min (K = 16, one MMA); the epilogue adds d_sb * (hi + lo) - dmin_sb * (hi + lo)
//     of the two into f32 registers.  d and dmin stay f32 outside the tensor core.
//
// CTA = 128 weight rows x all K (or a split of K), 13 warps, 4 smem stages of half a
// superblock:
//   warps 0-7   producers: dequantise the packed rows of half a superblock into the fp16 A
//               tile (core-matrix layout, no swizzle) and bulk-copy the prepared B tile
//   warp 8      MMA issuer: one thread issues tcgen05.mma, commits to mbarriers
//   warps 9-12  epilogue: tcgen05.ld of a region, scale, accumulate; then the output
// Every mbarrier wait is bounded; on a timeout the CTA records JDG_ERR_TIMEOUT, waits
// (bounded) for the copies and MMAs it issued, frees its tensor memory and returns.
#pragma once
#include <type_traits>

#include "jdg_hb1.cuh"

namespace jdg {

// ---------------------------------------------------------------------------------
// mbarriers and 1-D bulk async copies (TMA) into shared memory.  Every wait is bounded.
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// Wait for phase `parity` of bar with an iteration limit (try_wait also suspends for a
// bounded time per call); false when the limit ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    for (int it = 0; it < (1 << 20); it++) {
        uint32_t done;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
            : "=r"(done)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

constexpr int kQmRows = 128;            // weight rows per CTA (MMA M)
constexpr int kQmTok = 32;              // tokens (B rows 0..31 hi, 32..63 lo)
constexpr int kQmN = 2 * kQmTok;        // MMA N
constexpr int kQmStages = 4;            // smem stages, half a superblock (128 K) each
constexpr int kQmRegions = 4;           // TMEM regions (128 columns: 64 main + 64 min)
constexpr int kQmMaxSplit = 8;          // split-K ways at most
constexpr int kQmProd = 8;                      // producer warps
constexpr int kQmRowsPerProd = kQmRows / kQmProd;  // 16: two groups of 8 rows
constexpr int kQmMmaWarp = kQmProd;
constexpr int kQmThreads = (kQmProd + 5) * 32;
// prepared B per superblock in global memory: main 64 x 256 fp16, min 64 x 16
constexpr int kQmBMain = kQmN * 256 * 2;              // 32768
constexpr int kQmBMin = kQmN * 16 * 2;                // 2048
constexpr int kQmBBytes = kQmBMain + kQmBMin;
constexpr int kQmBHalf = kQmBMain / 2;                // the B main half a stage holds
// per stage: A main 128 x 128 fp16, A min 128 x 16, B main half 64 x 128, B min 64 x 16
constexpr int kQmAMain = kQmRows * 128 * 2;           // 32768
constexpr int kQmAMin = kQmRows * 16 * 2;             // 4096
constexpr int kQmStageBytes = kQmAMain + kQmAMin + kQmBHalf + kQmBMin;  // 55296
constexpr int kQmSmem = 1024 + kQmStages * kQmStageBytes;

// Core-matrix layout (K-major, no swizzle): 8 rows x 8 fp16 (16 bytes per row) = 128 bytes
// contiguous; core matrix (row group g, K chunk c) at (c * G + g) * 128 bytes, G = rows/8.
// Descriptor: LBO = K-chunk stride (G * 128), SBO = row-group stride (128).
__device__ __forceinline__ uint64_t qm_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);  // version 1, no swizzle
}
// kind::f16 instruction descriptor: D f32, A/B f16, both K-major, N = 64, M = 128
constexpr uint32_t kQmIdesc = (1u << 4) | ((uint32_t)(kQmN >> 3) << 17) | ((uint32_t)(kQmRows >> 4) << 24);

__device__ __forceinline__ void qm_mma(uint32_t dtmem, uint64_t da, uint64_t db, uint32_t acc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(dtmem),
        "l"(da), "l"(db), "r"(kQmIdesc), "r"(acc));
}
__device__ __forceinline__ void qm_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void qm_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void qm_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// 32 consecutive f32 columns of this warp's 32 TMEM lanes
__device__ __forceinline__ void qm_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void qm_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

struct QmArgs {
    QW w;                  // Q4_K, rows x cols (cols % 256 == 0)
    const uint8_t *xprep;  // prepared B: [cols/256][kQmBBytes]
    int M;                 // tokens (<= 32)
    float *C;              // C[t * ldc + n]
    int ldc;
    int epi;               // EPI_STORE, EPI_ADD (C += alpha * Y), EPI_SWIGLU (C[t][n/2] = silu(Y[2i]) * Y[2i+1])
    float alpha;
    int *err;
    // split-K: grid.y = ksplit CTAs share a row tile; partials [ksplit][32][rows] in `part`,
    // the last CTA of the tile (ticket) adds them in split order and applies the epilogue
    int ksplit;
    float *part;
    unsigned *tickets;
    // optional timeline of CTA (0,0) for tuning (%globaltimer ns): [0] entry, [1] exit,
    // [2 + 3i] producers done with superblock i, [3 + 3i] its MMAs issued, [4 + 3i] its
    // epilogue done, [194 + 2i] its B tile landed, [195 + 2i] its A tile complete (i < 64);
    // 322 entries
    unsigned long long *tl;
};

// X [M][K] f32 -> prepared B superblocks: fp16 hi/lo of x (rows 0..31 / 32..63, zero for
// t >= M) in the core-matrix layout, and of the 8 sub-block sums in B_min (K columns 0..7,
// the sums in f32 in index order).  grid (K/256), block 256: the 32 x 256 tile is staged in
// shared memory first.
static __global__ __launch_bounds__(256) void k_qm_prep_x(const float *__restrict__ X, int ldx, int M, int K,
                                                          uint8_t *__restrict__ out) {
    __shared__ float xt[kQmTok][257];
    __shared__ float sums[kQmTok][9];
    const int sb = blockIdx.x, tid = threadIdx.x;
    for (int t = 0; t < kQmTok; t++) xt[t][tid] = t < M ? X[(size_t)t * ldx + sb * 256 + tid] : 0.f;
    __syncthreads();
    {
        const int t = tid >> 3, j = tid & 7;
        float sm = 0.f;
        for (int i = 0; i < 32; i++) sm += xt[t][32 * j + i];
        sums[t][j] = sm;
    }
    uint8_t *o = out + (size_t)sb * kQmBBytes;
    // main: 64 rows x 32 chunks of 8
    for (int idx = tid; idx < kQmN * 32; idx += 256) {
        const int row = idx % kQmN, c = idx / kQmN, t = row % kQmTok;
        const bool lo = row >= kQmTok;
        uint32_t v[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float x0 = xt[t][c * 8 + 2 * i], x1 = xt[t][c * 8 + 2 * i + 1];
            const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
            const __half r0 = lo ? __float2half_rn(x0 - __half2float(h0)) : h0;
            const __half r1 = lo ? __float2half_rn(x1 - __half2float(h1)) : h1;
            v[i] = (uint32_t)__half_as_ushort(r0) | ((uint32_t)__half_as_ushort(r1) << 16);
        }
        *reinterpret_cast<uint4 *>(o + ((size_t)(c * (kQmN / 8) + row / 8) * 8 + row % 8) * 16) = make_uint4(v[0], v[1], v[2], v[3]);
    }
    __syncthreads();
    // min: 64 rows x 2 chunks; chunk 0 holds the 8 sub-block sums, chunk 1 zeros
    uint8_t *om = o + kQmBMain;
    if (tid < kQmN * 2) {
        const int row = tid % kQmN, c = tid / kQmN, t = row % kQmTok;
        const bool lo = row >= kQmTok;
        uint32_t v[4] = {0, 0, 0, 0};
        if (c == 0)
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float s0 = sums[t][2 * i], s1 = sums[t][2 * i + 1];
                const __half h0 = __float2half_rn(s0), h1 = __float2half_rn(s1);
                const __half r0 = lo ? __float2half_rn(s0 - __half2float(h0)) : h0;
                const __half r1 = lo ? __float2half_rn(s1 - __half2float(h1)) : h1;
                v[i] = (uint32_t)__half_as_ushort(r0) | ((uint32_t)__half_as_ushort(r1) << 16);
            }
        *reinterpret_cast<uint4 *>(om + ((size_t)(c * (kQmN / 8) + row / 8) * 8 + row % 8) * 16) = make_uint4(v[0], v[1], v[2], v[3]);
    }
}

// Byte i (0..15) of a 16-byte Q4_K superblock header held in registers.
__device__ __forceinline__ uint32_t hdr_byte(const uint4 &h, int i) {
    const uint32_t w = i < 4 ? h.x : i < 8 ? h.y : i < 12 ? h.z : h.w;
    return (w >> (8 * (i & 3))) & 0xFFu;
}
// jd_smk4 (janusdoe.c:2559-2561) on the header in registers: the 12 packed bytes are
// header bytes 4..15.
__device__ __forceinline__ void smk4_reg(int j, const uint4 &h, int &sc, int &mm) {
    if (j < 4) {
        sc = (int)(hdr_byte(h, 4 + j) & 63u);
        mm = (int)(hdr_byte(h, 8 + j) & 63u);
    } else {
        sc = (int)((hdr_byte(h, 8 + j) & 15u) | ((hdr_byte(h, j) >> 6) << 4));
        mm = (int)((hdr_byte(h, 8 + j) >> 4) | ((hdr_byte(h, 4 + j) >> 6) << 4));
    }
}
// Small non-negative integers (< 1024) as fp16 without the conversion unit: the half with
// bits 0x6400 | n is 1024 + n; subtracting 1024 is exact.
__device__ __forceinline__ __half2 small_int_h2(uint32_t a, uint32_t b) {
    const uint32_t v = (0x6400u | a) | ((0x6400u | b) << 16);
    return __hsub2(*reinterpret_cast<const __half2 *>(&v), __half2half2(__ushort_as_half(0x6400)));
}
__device__ __forceinline__ uint32_t half2_bits(int a, int b) {
    const __half2 h = small_int_h2((uint32_t)a, (uint32_t)b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Two 4-bit codes as an fp16 pair times the integer scale s, exactly: 0x6400 | v is the
// half 1024 + v, and fma((1024 + v), s, -1024 s) = v * s (<= 945) is exact in one rounding.
__device__ __forceinline__ uint32_t nib2_scaled(uint32_t pair, __half2 s2, __half2 bias) {
    const uint32_t hv = (pair & 0x000F000Fu) | 0x64006400u;
    const __half2 r = __hfma2(*reinterpret_cast<const __half2 *>(&hv), s2, bias);
    return *reinterpret_cast<const uint32_t *>(&r);
}

// Dequantise 16 code bytes (32 weights: 16 low nibbles of sub-block 2c at K positions
// k_lo.., 16 high nibbles of sub-block 2c+1 at k_hi..) into fp16 s*q values and store them
// as four 16-byte core-matrix rows.  Registers only.
__device__ __forceinline__ void qm_store_codes(uint8_t *A, int row, int k_lo, int k_hi, uint4 q, int s_lo, int s_hi) {
    const __half2 sl2 = small_int_h2((uint32_t)s_lo, (uint32_t)s_lo), sh2 = small_int_h2((uint32_t)s_hi, (uint32_t)s_hi);
    const __half2 m1024 = __half2half2(__ushort_as_half(0xE400));  // -1024
    const __half2 bl = __hmul2(sl2, m1024), bh = __hmul2(sh2, m1024);  // -1024 s, exact
    const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
    uint32_t lo[8], hi[8];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        // bytes (0,1) and (2,3) of the word into the two 16-bit halves
        const uint32_t p01 = __byte_perm(wd[i], 0, 0x4140), p23 = __byte_perm(wd[i], 0, 0x4342);
        lo[2 * i] = nib2_scaled(p01, sl2, bl);
        lo[2 * i + 1] = nib2_scaled(p23, sl2, bl);
        hi[2 * i] = nib2_scaled(p01 >> 4, sh2, bh);
        hi[2 * i + 1] = nib2_scaled(p23 >> 4, sh2, bh);
    }
    const int g = row >> 3, r0 = row & 7;
    constexpr int G = kQmRows / 8;
    const int c0 = k_lo >> 3, c1 = k_hi >> 3;
    *reinterpret_cast<uint4 *>(A + ((size_t)(c0 * G + g) * 8 + r0) * 16) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    *reinterpret_cast<uint4 *>(A + ((size_t)((c0 + 1) * G + g) * 8 + r0) * 16) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
    *reinterpret_cast<uint4 *>(A + ((size_t)(c1 * G + g) * 8 + r0) * 16) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4 *>(A + ((size_t)((c1 + 1) * G + g) * 8 + r0) * 16) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
}

// Output of one row n for the first a.M tokens (all lanes of the warp call it).
__device__ __forceinline__ void qm_epilogue(const QmArgs &a, const float (&acc)[kQmTok], int n, int lane) {
    if (a.epi == EPI_SWIGLU) {
        // rows 2i (gate) and 2i+1 (up) sit in adjacent lanes
#pragma unroll
        for (int t = 0; t < kQmTok; t++) {
            const float other = __shfl_xor_sync(JDG_FULL, acc[t], 1);
            if (!(lane & 1) && t < a.M && n + 1 < a.w.rows) a.C[(size_t)t * a.ldc + n / 2] = __fmul_rn(silu_ref(acc[t]), other);
        }
    } else if (n < a.w.rows) {
#pragma unroll
        for (int t = 0; t < kQmTok; t++) {
            if (t >= a.M) break;
            float *cp = a.C + (size_t)t * a.ldc + n;
            if (a.epi == EPI_ADD) *cp = __fadd_rn(*cp, __fmul_rn(acc[t], a.alpha));
            else *cp = acc[t];
        }
    }
}

// grid (rows/128, ksplit), block kQmThreads, dynamic smem kQmSmem.  One TMEM allocation of
// 512 columns.  Stage j holds half h = j % 2 of superblock i = j / 2 (K range 128h..128h+127);
// superblock i accumulates in TMEM region i % 4 over its two stages.
static __global__ __launch_bounds__(kQmThreads, 1) void k_qm_q4k(QmArgs a) {
    extern __shared__ __align__(1024) uint8_t qsm[];
    uint64_t *full_a = reinterpret_cast<uint64_t *>(qsm);        // [S] producers done (256 arrivals)
    uint64_t *full_b = full_a + kQmStages;                         // [S] B bulk copies landed
    uint64_t *empty = full_b + kQmStages;                          // [S] MMAs of the stage done
    uint64_t *ready = empty + kQmStages;                           // [R] region complete
    uint64_t *tfree = ready + kQmRegions;                          // [R] epilogue read the region (128 arrivals)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tfree + kQmRegions);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    uint8_t *stages = qsm + 1024;
    const bool tl_on = a.tl && blockIdx.x == 0 && blockIdx.y == 0;
    auto tl_mark = [&](int slot) {
        if (tl_on && slot < 2 + 5 * 64) {
            unsigned long long t;
            asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
            a.tl[slot] = t;
        }
    };
    if (threadIdx.x == 0) tl_mark(0);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = a.w.cols, nsb = K / 256, n0 = blockIdx.x * kQmRows;
    const int ks = a.ksplit > 1 ? a.ksplit : 1, kz = blockIdx.y, sb0 = (int)((long long)kz * nsb / ks);
    const int nloc = (int)((long long)(kz + 1) * nsb / ks) - sb0;  // superblocks of this CTA
    const int nst = 2 * nloc;                                       // stages of this CTA
    if (tid == 0) {
        for (int s = 0; s < kQmStages; s++) {
            mbar_init(&full_a[s], kQmProd * 32);
            mbar_init(&full_b[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int q = 0; q < kQmRegions; q++) {
            mbar_init(&ready[q], 1);
            mbar_init(&tfree[q], 128);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kQmMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    qm_fence_before();
    __syncthreads();
    qm_fence_after();
    const uint32_t tmem = *tmem_slot;
    int issued_mma = 0;  // stages whose MMAs were issued (lane 0 of the MMA warp)
    int issued_b = 0;    // stages whose B copies were issued (thread 0)

    if (warp < kQmProd) {
        // ---------------- producers ----------------
        // warp w owns rows 16w..16w+15 (2 groups of 8).  A row's half superblock is 64 code
        // bytes = 4 pieces of 16.  Pass p covers row group p: lane l takes row 8p + l%8 and
        // piece l/8, so the 8 lanes of a piece store one whole 128-byte core matrix (no bank
        // conflicts).  Raw loads run three stages ahead in a ring of register buffers.
        auto load_st = [&](int j, uint4 (&qv)[2], uint4 (&hv)[2]) {
            const int sb = sb0 + (j >> 1), piece = 4 * (j & 1) + (lane >> 3);
#pragma unroll
            for (int pass = 0; pass < 2; pass++) {
                const int n = n0 + warp * kQmRowsPerProd + pass * 8 + (lane & 7);
                qv[pass] = make_uint4(0, 0, 0, 0);
                hv[pass] = make_uint4(0, 0, 0, 0);
                if (j < nst && n < a.w.rows) {
                    qv[pass] = ld_stream_u4(a.w.q + (size_t)n * (K / 2) + (size_t)sb * 128 + piece * 16);
                    hv[pass] = ld_nc_u4(a.w.s + ((size_t)n * nsb + sb) * 16);
                }
            }
        };
        // H (the half, j % 2) is a compile-time constant: the scale bytes a lane needs then sit
        // at fixed header positions, two candidates per lane chosen by lane / 16
        auto produce = [&](int j, const uint4 (&qv)[2], const uint4 (&hv)[2], auto h_tag) -> bool {
            constexpr int h = decltype(h_tag)::value;
            const int s = j % kQmStages, sb = sb0 + (j >> 1);
            if (j >= kQmStages && !mbar_wait(&empty[s], (uint32_t)((j / kQmStages) - 1) & 1u)) *abort_flag = 1;
            if (*abort_flag) return false;
            if (tid == 0 && h == 1 && (j >> 1) < 64) tl_mark(2 + 3 * 64 + 2 * (j >> 1));  // producer starts half 1
            uint8_t *st = stages + (size_t)s * kQmStageBytes;
            uint8_t *Am = st, *An = st + kQmAMain, *Bm = An + kQmAMin, *Bn = Bm + kQmBHalf;
            if (tid == 0) {
                const uint8_t *src = a.xprep + (size_t)sb * kQmBBytes;
                mbar_expect_tx(&full_b[s], kQmBHalf + (h == 0 ? kQmBMin : 0));
                bulk_g2s(Bm, src + (size_t)h * kQmBHalf, kQmBHalf, &full_b[s]);
                if (h == 0) bulk_g2s(Bn, src + kQmBMain, kQmBMin, &full_b[s]);
                issued_b = j + 1;
            }
#pragma unroll
            for (int pass = 0; pass < 2; pass++) {
                const int row = warp * kQmRowsPerProd + pass * 8 + (lane & 7), piece = 4 * h + (lane >> 3);
                const int c = piece >> 1, l0 = (piece & 1) * 16;
                // sub-blocks 2c and 2c+1 with c = 2h + lane/16
                int sa, sbb, sc_, sd, mm;
                smk4_reg(4 * h, hv[pass], sa, mm);
                smk4_reg(4 * h + 1, hv[pass], sbb, mm);
                smk4_reg(4 * h + 2, hv[pass], sc_, mm);
                smk4_reg(4 * h + 3, hv[pass], sd, mm);
                const bool hiC = (lane >> 4) & 1;
                const int s0 = hiC ? sc_ : sa, s1 = hiC ? sd : sbb;
                qm_store_codes(Am, row, 64 * c + l0 - 128 * h, 64 * c + 32 + l0 - 128 * h, qv[pass], s0, s1);
                if (h == 0 && (lane >> 3) == 0) {
                    // A_min row: m_0..m_7 in K columns 0..7, zeros in 8..15
                    int mj[8];
#pragma unroll
                    for (int jj = 0; jj < 8; jj++) {
                        int sj;
                        smk4_reg(jj, hv[pass], sj, mj[jj]);
                    }
                    constexpr int G = kQmRows / 8;
                    const int g = row >> 3, r0 = row & 7;
                    *reinterpret_cast<uint4 *>(An + ((size_t)(0 * G + g) * 8 + r0) * 16) =
                        make_uint4(half2_bits(mj[0], mj[1]), half2_bits(mj[2], mj[3]), half2_bits(mj[4], mj[5]),
                                   half2_bits(mj[6], mj[7]));
                    *reinterpret_cast<uint4 *>(An + ((size_t)(1 * G + g) * 8 + r0) * 16) = make_uint4(0, 0, 0, 0);
                }
            }
            // generic-proxy stores must be visible to the tensor core (async proxy)
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(&full_a[s]);
            if (tid == 0 && h == 1) tl_mark(2 + 3 * (j >> 1));
            return true;
        };
        uint4 qa[2], ha[2], qb[2], hb[2], qc[2], hc[2], qd[2], hd[2];
        // weights do not depend on the previous kernel: the first stages load before the
        // dependency wait (Programmatic Dependent Launch)
        load_st(0, qa, ha);
        load_st(1, qb, hb);
        load_st(2, qc, hc);
        pdl_wait();
        pdl_trigger();
        using H0 = std::integral_constant<int, 0>;
        using H1 = std::integral_constant<int, 1>;
        for (int j = 0; j < nst; j += 4) {  // nst is even: j, j+2 are first halves
            load_st(j + 3, qd, hd);
            if (!produce(j, qa, ha, H0{}) || j + 1 >= nst) break;
            load_st(j + 4, qa, ha);
            if (!produce(j + 1, qb, hb, H1{}) || j + 2 >= nst) break;
            load_st(j + 5, qb, hb);
            if (!produce(j + 2, qc, hc, H0{}) || j + 3 >= nst) break;
            load_st(j + 6, qc, hc);
            if (!produce(j + 3, qd, hd, H1{})) break;
        }
    } else if (warp == kQmMmaWarp) {
        // ---------------- MMA issuer ----------------
        pdl_trigger();
        if (lane == 0) {
            constexpr int GA = kQmRows / 8, GB = kQmN / 8;
            for (int j = 0; j < nst; j++) {
                const int s = j % kQmStages, h = j & 1, i = j >> 1, q = i % kQmRegions;
                const uint32_t ph = (uint32_t)(j / kQmStages) & 1u;
                bool ok = mbar_wait(&full_b[s], ph);
                ok = ok && mbar_wait(&full_a[s], ph);
                if (h == 1 && i < 64) tl_mark(2 + 3 * 64 + 2 * i + 1);
                if (ok && h == 0 && i >= kQmRegions) ok = mbar_wait(&tfree[q], (uint32_t)((i / kQmRegions) - 1) & 1u);
                if (!ok || *abort_flag) {
                    *abort_flag = 1;
                    break;
                }
                qm_fence_after();
                const uint32_t st = smem_u32(stages + (size_t)s * kQmStageBytes);
                const uint32_t am = st, an = st + kQmAMain, bm = an + kQmAMin, bn = bm + kQmBHalf;
                const uint32_t dmain = tmem + (uint32_t)(q * 128), dmin = dmain + 64;
#pragma unroll
                for (int k8 = 0; k8 < 8; k8++)
                    qm_mma(dmain, qm_desc(am + k8 * 2 * GA * 128, GA * 128, 128), qm_desc(bm + k8 * 2 * GB * 128, GB * 128, 128),
                           (h > 0 || k8 > 0) ? 1u : 0u);
                if (h == 0) qm_mma(dmin, qm_desc(an, GA * 128, 128), qm_desc(bn, GB * 128, 128), 0);
                qm_commit(&empty[s]);
                if (h == 1) qm_commit(&ready[q]);
                issued_mma = j + 1;
                if (h == 1) tl_mark(3 + 3 * i);
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue: warps 9..12, TMEM lane quarter warp % 4 ----------------
        const int quarter = warp & 3, row = quarter * 32 + lane, n = n0 + row;
        pdl_wait();  // the epilogue reads and writes C
        pdl_trigger();
        float acc[kQmTok];
#pragma unroll
        for (int t = 0; t < kQmTok; t++) acc[t] = 0.f;
        // the superblock scales (d, dmin: the first 4 bytes of each header) are loaded one
        // superblock ahead, so their latency hides behind the wait for the region
        auto hdr_word = [&](int i) -> uint32_t {
            return (i < nloc && n < a.w.rows) ? __ldg(reinterpret_cast<const uint32_t *>(a.w.s + ((size_t)n * nsb + sb0 + i) * 16))
                                              : 0u;
        };
        uint32_t hw_next = hdr_word(0);
        for (int i = 0; i < nloc; i++) {
            const int q = i % kQmRegions;
            const uint32_t hw = hw_next;
            hw_next = hdr_word(i + 1);
            const bool ok = mbar_wait(&ready[q], (uint32_t)(i / kQmRegions) & 1u);
            if (!ok) *abort_flag = 1;
            // the TMEM loads below are warp-collective: leave the loop as a whole warp
            if (__any_sync(JDG_FULL, !ok || *abort_flag)) break;
            qm_fence_after();
            const uint32_t base = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(q * 128);
            float mh[32], ml[32];
            const float d = h2f((uint16_t)(hw & 0xFFFF)), dmin = h2f((uint16_t)(hw >> 16));
            qm_ld32(base, mh);
            qm_ld32(base + 32, ml);
            qm_ld_wait();
#pragma unroll
            for (int t = 0; t < kQmTok; t++) acc[t] = fmaf(d, mh[t] + ml[t], acc[t]);
            qm_ld32(base + 64, mh);
            qm_ld32(base + 96, ml);
            qm_ld_wait();
            qm_fence_before();
            mbar_arrive(&tfree[q]);
            if (warp == kQmMmaWarp + 1 && lane == 0) tl_mark(4 + 3 * i);
#pragma unroll
            for (int t = 0; t < kQmTok; t++) acc[t] = fmaf(-dmin, mh[t] + ml[t], acc[t]);
        }
        if (!__any_sync(JDG_FULL, *abort_flag)) {
            if (ks == 1) {
                qm_epilogue(a, acc, n, lane);
            } else if (n < a.w.rows) {
#pragma unroll
                for (int t = 0; t < kQmTok; t++) {
                    if (t >= a.M) break;
                    a.part[((size_t)kz * kQmTok + t) * a.w.rows + n] = acc[t];
                }
            }
        }
    }
    __syncthreads();
    if (ks > 1 && !*abort_flag) {
        // the last CTA of this row tile adds the partials in split order
        __shared__ unsigned s_last;
        if (tid == 0) {
            __threadfence();
            const unsigned t = atomicAdd(a.tickets + blockIdx.x, 1u);
            s_last = t == (unsigned)ks - 1;
            if (s_last) {
                __threadfence();
                a.tickets[blockIdx.x] = 0;
            }
        }
        __syncthreads();
        if (s_last && warp > kQmMmaWarp) {
            const int row = (warp & 3) * 32 + lane, n = n0 + row;
            float acc[kQmTok];
#pragma unroll
            for (int t = 0; t < kQmTok; t++) acc[t] = 0.f;
            // split by split, all tokens' loads in flight at once (ks round trips in total)
            for (int z = 0; z < ks; z++) {
                float v[kQmTok];
#pragma unroll
                for (int t = 0; t < kQmTok; t++)
                    v[t] = (t < a.M && n < a.w.rows) ? __ldcg(a.part + ((size_t)z * kQmTok + t) * a.w.rows + n) : 0.f;
#pragma unroll
                for (int t = 0; t < kQmTok; t++) acc[t] += v[t];
            }
            qm_epilogue(a, acc, n, lane);
        }
    }
    if (*abort_flag) {
        if (tid == 0) atomicOr(a.err, JDG_ERR_TIMEOUT);
        // let the issued MMAs and copies land before the memory goes away
        if (warp == kQmMmaWarp && lane == 0 && issued_mma > 0) {
            const int j = issued_mma - 1;
            mbar_wait(&empty[j % kQmStages], (uint32_t)(j / kQmStages) & 1u);
        }
        if (tid == 0)
            for (int j = max(0, issued_b - kQmStages); j < issued_b; j++)
                mbar_wait(&full_b[j % kQmStages], (uint32_t)(j / kQmStages) & 1u);
    }
    qm_fence_before();
    __syncthreads();
    if (warp == kQmMmaWarp) {
        qm_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
    if (threadIdx.x == 0) tl_mark(1);
}

}  // namespace jdg

// jdg_qmma.cuh — batched host GEMM over Q4_K weights on the 5th-generation tensor cores
// (tcgen05.mma with the A operand in tensor memory), for the host GGUF path at batch > 1.
//
//   Y[t][n] (epi)= sum_k X[t][k] * W[n][k],   W in Q4_K (janusdoe.c:2573-2585):
//   W[n][k] = d_sb * s_j * q - dmin_sb * m_j   (superblock sb of 256 weights, sub-block j of 32)
//
// Exact reformulation on fp16 tensor cores with f32 accumulation:
//   * A = s_j * q is an integer <= 63 * 15 = 945: exact in fp16.
//   * X is split into x_hi = fp16(x) and x_lo = fp16(x - x_hi); together they carry ~22
//     mantissa bits.  B stacks them as 64 "columns": tokens 0..31 hi, then 0..31 lo.
//   * The sub-block minimum becomes a second product against the sums of x over each
//     sub-block, split hi/lo along K: A_min[n] = (m_0..m_7, m_0..m_7) (integers <= 63),
//     B_min[t] = (sum_hi_0..7, sum_lo_0..7), one 128x32x16 MMA.
//   * Per superblock one TMEM region receives A.B (K = 256: 16 MMAs of 128x64x16) and
//     A_min.B_min; the epilogue adds d_sb * (hi + lo) - dmin_sb * min into f32 registers.
//     d and dmin stay f32 outside the tensor core.
//
// CTA = 128 weight rows x all K (or a split of K), 23 warps:
//   warps 0-15   producers: warp w fills TMEM lanes 32(w%4).. (its 32 rows, one per lane) for
//                the K quarter w/4 of each superblock: it reads the raw codes from shared
//                memory, forms the fp16 s*q pairs and stores them with tcgen05.st; warps 0-3
//                also write the A_min rows into shared memory
//   warps 16-17  MMA issuers (one thread each): warp 16 the even superblocks, warp 17 the odd
//                ones; their smem stages, A stages and accumulator regions are disjoint, so the
//                two streams of MMAs need no ordering (one thread issues ~1 MMA per 50 cycles)
//   warp 18      TMA issuer (one thread): per superblock the code bytes (128 rows x 128 B,
//                128-byte swizzle), the headers (128 x 16 B) and the prepared B tile (34 KB)
//   warps 19-22  epilogue (TMEM lane quarter warp % 4)
// Shared memory: kQmStages stages of one superblock.  TMEM (512 columns): five A stages of
// half a superblock (64 columns: K 128 as fp16 pairs; warps w/4 = 2h, 2h+1 fill half h) and
// two accumulator regions of 96 columns (A.B 64, A_min.B_min 32).
// Every mbarrier wait is bounded; on a timeout the CTA records JDG_ERR_TIMEOUT, waits
// (bounded) for the copies and MMAs it issued, frees its tensor memory and returns.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <type_traits>

#include "jdg_async.cuh"
#include "jdg_hb1.cuh"

namespace jdg {

constexpr int kQmRows = 128;             // weight rows per CTA (MMA M)
constexpr int kQmTok = 32;               // tokens (B rows 0..31 hi, 32..63 lo)
constexpr int kQmN = 2 * kQmTok;         // MMA N
constexpr int kQmStages = 4;             // shared-memory stages, one superblock each
constexpr int kQmAStages = 5;            // TMEM A stages of half a superblock (64 columns)
constexpr int kQmRegions = 2;            // TMEM accumulator regions (96 columns)
constexpr int kQmRegionCols = 96;
constexpr int kQmMaxSplit = 8;           // split-K ways at most
constexpr int kQmProd = 16;              // producer warps
constexpr int kQmMmaWarp = 16, kQmTmaWarp = 18;  // MMA issuers: warps 16, 17
constexpr int kQmThreads = 23 * 32;
constexpr int kQmCodes = kQmRows * 128;  // code bytes of one superblock
constexpr int kQmHdr = kQmRows * 16;     // headers of one superblock
constexpr int kQmAMin = kQmRows * 16 * 2;    // A_min of one superblock (fp16, core-matrix layout)
constexpr int kQmBMain = kQmN * 256 * 2;     // B tile of one superblock (fp16, core-matrix layout)
constexpr int kQmBMin = kQmTok * 16 * 2;     // B_min: hi/lo of the sub-block sums along K
constexpr int kQmBBytes = kQmBMain + kQmBMin;  // prepared activations per superblock in global memory
constexpr int kQmStageBytes = kQmCodes + kQmHdr + kQmAMin + kQmBBytes;  // 56320 = 55 KB
constexpr int kQmSmem = 1024 + kQmStages * kQmStageBytes;
constexpr uint32_t kQmRegionCol = kQmAStages * 64;  // first accumulator column
static_assert(kQmRegionCol + kQmRegions * kQmRegionCols <= 512, "TMEM columns");

// Core-matrix layout (K-major, no swizzle): 8 rows x 8 fp16 (16 bytes per row) = 128 bytes
// contiguous; core matrix (row group g, K chunk c) at (c * G + g) * 128 bytes, G = rows/8.
// Descriptor: LBO = K-chunk stride (G * 128), SBO = row-group stride (128).
__device__ __forceinline__ uint64_t qm_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);  // version 1, no swizzle
}
// kind::f16 instruction descriptors: D f32, A/B f16, both K-major, M = 128, N = 64 (main) or
// 32 (minimum)
constexpr uint32_t kQmIdesc = (1u << 4) | ((uint32_t)(kQmN >> 3) << 17) | ((uint32_t)(kQmRows >> 4) << 24);
constexpr uint32_t kQmIdescMin = (1u << 4) | ((uint32_t)(kQmTok >> 3) << 17) | ((uint32_t)(kQmRows >> 4) << 24);

// tcgen05.mma with A in tensor memory (lane = row, K as fp16 pairs along the columns) and B
// from a shared-memory descriptor
__device__ __forceinline__ void qm_mma_ts(uint32_t dtmem, uint32_t atmem, uint64_t db, uint32_t acc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }" ::"r"(dtmem),
        "r"(atmem), "l"(db), "r"(kQmIdesc), "r"(acc));
}
// tcgen05.mma with A and B from shared-memory descriptors (the 128x32x16 minimum product)
__device__ __forceinline__ void qm_mma_min(uint32_t dtmem, uint64_t da, uint64_t db) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %3, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %4, p; }" ::"r"(dtmem),
        "l"(da), "l"(db), "r"(0), "r"(kQmIdescMin));
}
__device__ __forceinline__ void qm_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void qm_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void qm_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
// 8 consecutive f32 columns of this warp's 32 TMEM lanes
__device__ __forceinline__ void qm_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void qm_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 32 consecutive 32-bit TMEM columns of this warp's 32 lanes
__device__ __forceinline__ void qm_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// TMA tensor maps of one Q4_K matrix (made on the host with cuTensorMapEncodeTiled)
struct QmMaps {
    const uint8_t *q;  // the matrix's code bytes (identifies it)
    CUtensorMap codes, hdr;
};

struct QmArgs {
    QW w;                  // Q4_K, rows x cols (cols % 256 == 0)
    const uint8_t *xprep;  // prepared activations: [cols/256][kQmBBytes]
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
};

// K order inside the tensor-core tiles: within every group of 4 consecutive K positions the
// middle two are swapped (MMA position p holds source k = qm_kperm(p); the map is its own
// inverse).  A 32-bit word of 4 code bytes then yields its fp16 pairs (byte 0, byte 2) and
// (byte 1, byte 3) with one mask each, see qm_decode_word.
__host__ __device__ __forceinline__ int qm_kperm(int p) { return (p & ~3) | ((p & 1) << 1) | ((p >> 1) & 1); }

// fp16 hi/lo of an f32 pair, packed: the lo row of a B tile holds fp16(v - fp16(v))
__device__ __forceinline__ uint32_t qm_split2(float v0, float v1, bool lo) {
    const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
    const __half r0 = lo ? __float2half_rn(v0 - __half2float(h0)) : h0;
    const __half r1 = lo ? __float2half_rn(v1 - __half2float(h1)) : h1;
    return (uint32_t)__half_as_ushort(r0) | ((uint32_t)__half_as_ushort(r1) << 16);
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
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<const uint32_t *>(&h); }
__device__ __forceinline__ uint32_t half2_bits(int a, int b) { return h2_bits(small_int_h2((uint32_t)a, (uint32_t)b)); }
__device__ __forceinline__ __half2 bits_h2(uint32_t v) { return *reinterpret_cast<const __half2 *>(&v); }

// Scale constants of one sub-block for qm_decode_word.  Low nibbles: 0x6400 | q is the half
// 1024 + q and fma(1024 + q, s, -1024 s) = q s exactly (<= 945).  High nibbles stay in bits
// 4..7: 0x6400 | 16q is 1024 + 16 q and fma(1024 + 16 q, s / 16, -64 s) = q s exactly (s / 16
// is exact in fp16).
struct QmScale {
    __half2 s, b;
};
__device__ __forceinline__ QmScale qm_scale_lo(int s) {
    const __half2 s2 = small_int_h2((uint32_t)s, (uint32_t)s);
    return {s2, __hmul2(s2, __half2half2(__ushort_as_half(0xE400)))};  // -1024 s
}
__device__ __forceinline__ QmScale qm_scale_hi(int s) {
    const __half2 s2 = __hmul2(small_int_h2((uint32_t)s, (uint32_t)s), __half2half2(__ushort_as_half(0x2C00)));  // s/16
    return {s2, __hmul2(s2, __half2half2(__ushort_as_half(0xE400)))};  // -64 s
}
// 4 code bytes (K positions l..l+3 of two sub-blocks) -> 4 fp16 pairs in tensor-core K order:
// lo0 = (b0, b2), lo1 = (b1, b3) of the low nibbles, hi0, hi1 the same for the high nibbles.
__device__ __forceinline__ void qm_decode_word(uint32_t w, const QmScale &sl, const QmScale &sh, uint32_t &lo0,
                                               uint32_t &lo1, uint32_t &hi0, uint32_t &hi1) {
    const uint32_t w8 = w >> 8;
    lo0 = h2_bits(__hfma2(bits_h2((w & 0x000F000Fu) | 0x64006400u), sl.s, sl.b));
    lo1 = h2_bits(__hfma2(bits_h2((w8 & 0x000F000Fu) | 0x64006400u), sl.s, sl.b));
    hi0 = h2_bits(__hfma2(bits_h2((w & 0x00F000F0u) | 0x64006400u), sh.s, sh.b));
    hi1 = h2_bits(__hfma2(bits_h2((w8 & 0x00F000F0u) | 0x64006400u), sh.s, sh.b));
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
    } else if (n < a.w.rows && a.epi == EPI_ADD) {
        // eight tokens' C values loaded before any store (a load after a store to another
        // token's row could not be moved ahead of it: one L2 round trip per token)
#pragma unroll
        for (int t0 = 0; t0 < kQmTok; t0 += 8) {
            float c[8];
#pragma unroll
            for (int t = 0; t < 8; t++) c[t] = t0 + t < a.M ? a.C[(size_t)(t0 + t) * a.ldc + n] : 0.f;
#pragma unroll
            for (int t = 0; t < 8; t++)
                if (t0 + t < a.M) a.C[(size_t)(t0 + t) * a.ldc + n] = __fadd_rn(c[t], __fmul_rn(acc[t0 + t], a.alpha));
        }
    } else if (n < a.w.rows) {
#pragma unroll
        for (int t = 0; t < kQmTok; t++) {
            if (t >= a.M) break;
            a.C[(size_t)t * a.ldc + n] = acc[t];
        }
    }
}

// The same for tokens t0 .. t0 + 7 only (the split-K sum, where each warp owns eight tokens).
__device__ __forceinline__ void qm_epilogue8(const QmArgs &a, const float (&acc)[8], int t0, int n, int lane) {
    if (a.epi == EPI_SWIGLU) {
#pragma unroll
        for (int t = 0; t < 8; t++) {
            const float other = __shfl_xor_sync(JDG_FULL, acc[t], 1);
            if (!(lane & 1) && t0 + t < a.M && n + 1 < a.w.rows)
                a.C[(size_t)(t0 + t) * a.ldc + n / 2] = __fmul_rn(silu_ref(acc[t]), other);
        }
    } else if (n < a.w.rows && a.epi == EPI_ADD) {
        float c[8];
#pragma unroll
        for (int t = 0; t < 8; t++) c[t] = t0 + t < a.M ? a.C[(size_t)(t0 + t) * a.ldc + n] : 0.f;
#pragma unroll
        for (int t = 0; t < 8; t++)
            if (t0 + t < a.M) a.C[(size_t)(t0 + t) * a.ldc + n] = __fadd_rn(c[t], __fmul_rn(acc[t], a.alpha));
    } else if (n < a.w.rows) {
#pragma unroll
        for (int t = 0; t < 8; t++)
            if (t0 + t < a.M) a.C[(size_t)(t0 + t) * a.ldc + n] = acc[t];
    }
}

// grid (rows/128, ksplit), block kQmThreads, dynamic smem kQmSmem.  tm_codes: 2-D map over
// the code bytes [rows][cols/2], box 128 bytes x 128 rows, 128-byte swizzle; tm_hdr: 2-D map
// over the headers [rows][cols/256 * 16], box 16 bytes x 128 rows.  Rows past the end read
// as zeros.  One TMEM allocation of 512 columns.
static __global__ __launch_bounds__(kQmThreads, 1) void k_qm_q4k(QmArgs a, const __grid_constant__ CUtensorMap tm_codes,
                                                                const __grid_constant__ CUtensorMap tm_hdr) {
    extern __shared__ __align__(1024) uint8_t qsm[];
    uint64_t *rawf = reinterpret_cast<uint64_t *>(qsm);  // [S] codes + headers landed
    uint64_t *bf = rawf + kQmStages;                      // [S] B landed
    uint64_t *empty = bf + kQmStages;                     // [S] MMAs of the stage done
    uint64_t *a_full = empty + kQmStages;                 // [AS] A stage written (one arrival per producer warp of the half)
    uint64_t *a_empty = a_full + kQmAStages;              // [AS] MMAs that read the A stage done
    uint64_t *ready = a_empty + kQmAStages;               // [R] region complete
    uint64_t *tfree = ready + kQmRegions;                 // [R] epilogue read the region (one arrival per warp)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tfree + kQmRegions);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    uint8_t *stages = qsm + 1024;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // the 128-byte-swizzled TMA destinations need 1024-byte alignment
    if (smem_u32(qsm) & 1023u) {
        if (tid == 0) atomicOr(a.err, JDG_ERR_SHAPE);
        return;
    }
    const int K = a.w.cols, nsb = K / 256, n0 = blockIdx.x * kQmRows;
    const int ks = a.ksplit > 1 ? a.ksplit : 1, kz = blockIdx.y, sb0 = (int)((long long)kz * nsb / ks);
    const int nloc = (int)((long long)(kz + 1) * nsb / ks) - sb0;  // superblocks of this CTA
    if (tid == 0) {
        for (int s = 0; s < kQmStages; s++) {
            mbar_init(&rawf[s], 1);
            mbar_init(&bf[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < kQmAStages; s++) {
            mbar_init(&a_full[s], kQmProd / 2);
            mbar_init(&a_empty[s], 1);
        }
        for (int q = 0; q < kQmRegions; q++) {
            mbar_init(&ready[q], 1);
            mbar_init(&tfree[q], 4);
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
    int issued_mma = 0;  // A stages (half superblocks) whose MMAs were issued (MMA thread)
    int issued_ld = 0;   // superblocks whose copies were issued (TMA thread)

    if (warp < kQmProd) {
        // ---------------- producers ----------------
        pdl_trigger();
        const int quarter = warp & 3, kq = warp >> 2, row = quarter * 32 + lane;
        const uint32_t tlane = (uint32_t)(quarter * 32) << 16;
        // K quarter kq of a superblock = code bytes 32kq..32kq+31 of the row (16-byte chunks
        // 2kq, 2kq+1): low nibbles are sub-block 2kq, high nibbles sub-block 2kq+1.  It lies in
        // half h = kq / 2, columns 32 (kq % 2) of that half's A stage.
        auto body = [&](auto kq_tag) {
            constexpr int KQ = decltype(kq_tag)::value, H = KQ >> 1;
            for (int i = 0; i < nloc; i++) {
                const int s = i % kQmStages, j = 2 * i + H, as = j % kQmAStages;
                bool ok = mbar_wait(&rawf[s], (uint32_t)(i / kQmStages) & 1u);
                if (ok && j >= kQmAStages) ok = mbar_wait(&a_empty[as], (uint32_t)((j / kQmAStages) - 1) & 1u);
                if (!ok) *abort_flag = 1;
                // tcgen05.st is warp-collective: leave as a whole warp
                if (__any_sync(JDG_FULL, !ok || *abort_flag)) break;
                uint8_t *st = stages + (size_t)s * kQmStageBytes;
                const uint4 hv = *reinterpret_cast<const uint4 *>(st + kQmCodes + row * 16);
                const uint8_t *crow = st + row * 128;
                const uint4 c0 = *reinterpret_cast<const uint4 *>(crow + (((2 * KQ) ^ (row & 7)) << 4));
                const uint4 c1 = *reinterpret_cast<const uint4 *>(crow + (((2 * KQ + 1) ^ (row & 7)) << 4));
                int s_lo, s_hi, mm;
                smk4_reg(2 * KQ, hv, s_lo, mm);
                smk4_reg(2 * KQ + 1, hv, s_hi, mm);
                const QmScale sl = qm_scale_lo(s_lo), sh = qm_scale_hi(s_hi);
                // columns [0, 8) chunk 0 low, [8, 16) chunk 1 low, [16, 24) chunk 0 high,
                // [24, 32) chunk 1 high
                uint32_t r[32];
                const uint32_t w0[4] = {c0.x, c0.y, c0.z, c0.w}, w1[4] = {c1.x, c1.y, c1.z, c1.w};
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    qm_decode_word(w0[k], sl, sh, r[2 * k], r[2 * k + 1], r[16 + 2 * k], r[16 + 2 * k + 1]);
                    qm_decode_word(w1[k], sl, sh, r[8 + 2 * k], r[8 + 2 * k + 1], r[24 + 2 * k], r[24 + 2 * k + 1]);
                }
                qm_st32(tmem + tlane + (uint32_t)(as * 64 + (KQ & 1) * 32), r);
                if (KQ == 0) {
                    // A_min row: m_0..m_7 in K columns 0..7 and again in 8..15 (core-matrix layout)
                    int mj[8];
#pragma unroll
                    for (int jj = 0; jj < 8; jj++) {
                        int sj;
                        smk4_reg(jj, hv, sj, mj[jj]);
                    }
                    constexpr int G = kQmRows / 8;
                    uint8_t *An = st + kQmCodes + kQmHdr;
                    const int g = row >> 3, r0 = row & 7;
                    const uint4 mrow = make_uint4(half2_bits(mj[0], mj[1]), half2_bits(mj[2], mj[3]),
                                                  half2_bits(mj[4], mj[5]), half2_bits(mj[6], mj[7]));
                    *reinterpret_cast<uint4 *>(An + ((size_t)(0 * G + g) * 8 + r0) * 16) = mrow;
                    *reinterpret_cast<uint4 *>(An + ((size_t)(1 * G + g) * 8 + r0) * 16) = mrow;
                    // generic-proxy stores must be visible to the tensor core (async proxy)
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                }
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                qm_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&a_full[as]);
            }
        };
        switch (kq) {
        case 0: body(std::integral_constant<int, 0>{}); break;
        case 1: body(std::integral_constant<int, 1>{}); break;
        case 2: body(std::integral_constant<int, 2>{}); break;
        default: body(std::integral_constant<int, 3>{}); break;
        }
    } else if (warp < kQmTmaWarp) {
        // ---------------- MMA issuers: superblocks i with i % 2 == warp - kQmMmaWarp ----------------
        pdl_trigger();
        if (lane == 0) {
            constexpr int GA = kQmRows / 8, GB = kQmN / 8, GBM = kQmTok / 8;
            for (int j = 2 * (warp - kQmMmaWarp); j < 2 * nloc; j += (j & 1) ? 3 : 1) {
                const int i = j >> 1, h = j & 1, s = i % kQmStages, as = j % kQmAStages, q = i % kQmRegions;
                bool ok = true;
                if (h == 0) {
                    ok = mbar_wait(&bf[s], (uint32_t)(i / kQmStages) & 1u);
                    if (ok && i >= kQmRegions) ok = mbar_wait(&tfree[q], (uint32_t)((i / kQmRegions) - 1) & 1u);
                }
                ok = ok && mbar_wait(&a_full[as], (uint32_t)(j / kQmAStages) & 1u);
                if (!ok || *abort_flag) {
                    *abort_flag = 1;
                    break;
                }
                qm_fence_after();
                const uint32_t st = smem_u32(stages + (size_t)s * kQmStageBytes);
                const uint32_t an = st + kQmCodes + kQmHdr, bm = an + kQmAMin, bn = bm + kQmBMain;
                const uint32_t at = tmem + (uint32_t)(as * 64), dmain = tmem + kQmRegionCol + (uint32_t)(q * kQmRegionCols);
#pragma unroll
                for (int k = 0; k < 8; k++)
                    qm_mma_ts(dmain, at + (uint32_t)(8 * k), qm_desc(bm + (8 * h + k) * 2 * GB * 128, GB * 128, 128),
                              (h > 0 || k > 0) ? 1u : 0u);
                if (h == 0) qm_mma_min(dmain + 64, qm_desc(an, GA * 128, 128), qm_desc(bn, GBM * 128, 128));
                if (h == 1) {
                    qm_commit(&empty[s]);
                    qm_commit(&ready[q]);
                }
                qm_commit(&a_empty[as]);
                issued_mma = j + 1;
            }
        }
        __syncwarp();
    } else if (warp == kQmTmaWarp) {
        // ---------------- TMA issuer ----------------
        pdl_trigger();
        if (lane == 0) {
            auto raw = [&](int i) {
                const int s = i % kQmStages;
                uint8_t *st = stages + (size_t)s * kQmStageBytes;
                mbar_expect_tx(&rawf[s], kQmCodes + kQmHdr);
                tma_load_2d(st, &tm_codes, (sb0 + i) * 128, n0, &rawf[s]);
                tma_load_2d(st + kQmCodes, &tm_hdr, (sb0 + i) * 16, n0, &rawf[s]);
            };
            auto bload = [&](int i) {
                const int s = i % kQmStages;
                uint8_t *st = stages + (size_t)s * kQmStageBytes;
                mbar_expect_tx(&bf[s], kQmBBytes);
                bulk_g2s(st + kQmCodes + kQmHdr + kQmAMin, a.xprep + (size_t)(sb0 + i) * kQmBBytes, kQmBBytes, &bf[s]);
            };
            const int pre = nloc < kQmStages ? nloc : kQmStages;
            // the weights do not depend on the previous kernel: they load before the wait
            for (int i = 0; i < pre; i++) raw(i);
            pdl_wait();
            for (int i = 0; i < pre; i++) bload(i);
            issued_ld = pre;
            for (int i = pre; i < nloc; i++) {
                const int s = i % kQmStages;
                if (!mbar_wait(&empty[s], (uint32_t)((i / kQmStages) - 1) & 1u) || *abort_flag) {
                    *abort_flag = 1;
                    break;
                }
                raw(i);
                bload(i);
                issued_ld = i + 1;
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue: warps 19..22, TMEM lane quarter warp % 4 ----------------
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
            const uint32_t base = tmem + ((uint32_t)(quarter * 32) << 16) + kQmRegionCol + (uint32_t)(q * kQmRegionCols);
            const float d = h2f((uint16_t)(hw & 0xFFFF)), dmin = h2f((uint16_t)(hw >> 16));
#pragma unroll
            for (int qt = 0; qt < 4; qt++) {  // A.B: tokens 8qt.. hi and lo, then A_min.B_min
                float vh[8], vl[8], vm[8];
                qm_ld8(base + 8 * qt, vh);
                qm_ld8(base + 32 + 8 * qt, vl);
                qm_ld8(base + 64 + 8 * qt, vm);
                qm_ld_wait();
#pragma unroll
                for (int t = 0; t < 8; t++) {
                    acc[8 * qt + t] = fmaf(d, vh[t] + vl[t], acc[8 * qt + t]);
                    acc[8 * qt + t] = fmaf(-dmin, vm[t], acc[8 * qt + t]);
                }
            }
            qm_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tfree[q]);
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
        if (s_last && warp < 16) {
            // sixteen warps: TMEM-row quarter warp % 4, tokens 8 (warp / 4) .. + 7; four
            // splits' loads in flight at once, added in split order
            const int row = (warp & 3) * 32 + lane, n = n0 + row, t0 = 8 * (warp >> 2);
            float acc[8];
#pragma unroll
            for (int t = 0; t < 8; t++) acc[t] = 0.f;
            for (int z0 = 0; z0 < ks; z0 += 4) {
                float v[4][8];
#pragma unroll
                for (int zz = 0; zz < 4; zz++)
#pragma unroll
                    for (int t = 0; t < 8; t++)
                        v[zz][t] = (z0 + zz < ks && t0 + t < a.M && n < a.w.rows)
                                       ? __ldcg(a.part + ((size_t)(z0 + zz) * kQmTok + t0 + t) * a.w.rows + n)
                                       : 0.f;
#pragma unroll
                for (int zz = 0; zz < 4; zz++)
                    if (z0 + zz < ks)
#pragma unroll
                        for (int t = 0; t < 8; t++) acc[t] += v[zz][t];
            }
            qm_epilogue8(a, acc, t0, n, lane);
        }
    }
    if (*abort_flag) {
        if (tid == 0) atomicOr(a.err, JDG_ERR_TIMEOUT);
        // let the issued MMAs and copies land before the memory goes away
        if (warp >= kQmMmaWarp && warp < kQmTmaWarp && lane == 0 && issued_mma > 0) {
            const int j = issued_mma - 1;  // its commit follows every MMA issued before
            mbar_wait(&a_empty[j % kQmAStages], (uint32_t)(j / kQmAStages) & 1u);
        }
        if (warp == kQmTmaWarp && lane == 0)
            for (int i = max(0, issued_ld - kQmStages); i < issued_ld; i++) {
                mbar_wait(&rawf[i % kQmStages], (uint32_t)(i / kQmStages) & 1u);
                mbar_wait(&bf[i % kQmStages], (uint32_t)(i / kQmStages) & 1u);
            }
    }
    qm_fence_before();
    __syncthreads();
    if (warp == kQmMmaWarp) {
        qm_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}

}  // namespace jdg

/*
 * jd_quant.h — GGUF block formats: field extraction shared by the loader (C, host) and the
 * packed-weight kernels (CUDA, device), plus a table-driven whole-tensor decoder.
 *
 * Formats (GGML block layouts, little endian; the reference decodes the same layouts in
 * janusdoe.c:2545-2617):
 *   F16   2 B / weight, IEEE binary16.
 *   Q4_0  18 B / 32:  f16 d | 16 B of nibbles. Weight i<16 is the low nibble of byte i,
 *                     weight 16+i the high nibble; value (q - 8) * d.
 *   Q5_0  22 B / 32:  f16 d | u32 fifth bits | 16 B of nibbles; weight w takes bit w of
 *                     the u32 as its fifth bit; value (q - 16) * d.
 *   Q8_0  34 B / 32:  f16 d | 32 int8; value q * d.
 *   Q4_K  144 B / 256: f16 d | f16 dmin | 12 B of 6-bit (scale, min) pairs for 8 sub-blocks
 *                     of 32 | 128 B of nibbles. Sub-block j lives in code bytes
 *                     32*(j/2) .. +31, low nibbles for even j, high for odd j;
 *                     value (d*scale_j) * q - (dmin*min_j).
 *   Q6_K  210 B / 256: 128 B low nibbles | 64 B of 2-bit high parts | 16 int8 scales |
 *                     f16 d. Two halves of 128 weights; in a half, quarter u (32 weights)
 *                     takes its low nibble from byte l + 32*(u&1) of the half's 64 low bytes
 *                     (high nibble when u >= 2), its high 2 bits from bits 2u..2u+1 of the
 *                     half's byte l of the 32 high bytes, and scale 8*half + l/16 + 2u;
 *                     value (d*scale) * (q - 32).
 * The floating-point expressions are written in the order the values must be evaluated for
 * the decoded weights to be bit-identical to the reference's.
 */
#pragma once
#include <stdint.h>
#include <string.h>

#ifdef __CUDACC__
#define JDQ_FN static __host__ __device__ __forceinline__
#else
#define JDQ_FN static inline
#endif

/* IEEE binary16 -> binary32 (exact). Normal numbers re-bias the exponent (15 -> 127);
 * subnormals are mant * 2^-24, which binary32 represents exactly; exponent 31 is inf/nan
 * with the payload kept in the top mantissa bits. */
JDQ_FN float jdq_half(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, ex = (h >> 10) & 0x1Fu, mant = h & 0x3FFu, bits;
    if (ex == 0) {
        float v = (float)mant * 5.9604644775390625e-8f; /* 2^-24 */
        memcpy(&bits, &v, 4);
        bits |= sign;
    } else if (ex == 0x1Fu) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else {
        bits = sign | ((ex + 112u) << 23) | (mant << 13);
    }
    float r;
    memcpy(&r, &bits, 4);
    return r;
}
JDQ_FN float jdq_half_at(const uint8_t *p) { return jdq_half((uint16_t)(p[0] | (p[1] << 8))); }

/* Q4_K: 6-bit scale and minimum of sub-block j (0..7) from the 12 packed bytes p.
 * Bytes 0-3 hold scales 0-3 in their low 6 bits, bytes 4-7 minima 0-3; for sub-blocks 4-7
 * the low 4 bits come from the nibbles of bytes 8-11 (scale low, minimum high) and the top
 * 2 bits from bits 6-7 of bytes 0-3 (scale) and 4-7 (minimum). */
JDQ_FN void jdq_q4k_scale_min(const uint8_t *p, int j, int *s, int *m) {
    if (j < 4) {
        *s = p[j] & 0x3F;
        *m = p[4 + j] & 0x3F;
    } else {
        const int i = j - 4;
        *s = (p[8 + i] & 0x0F) | ((p[i] & 0xC0) >> 2);
        *m = (p[8 + i] >> 4) | ((p[4 + i] & 0xC0) >> 2);
    }
}

#ifndef __CUDACC__
/* ---- whole-tensor decoding (host) ---- */
static void jdq_block_f16(const uint8_t *b, float *y) { y[0] = jdq_half_at(b); }

static void jdq_block_q4_0(const uint8_t *b, float *y) {
    const float d = jdq_half_at(b);
    for (int w = 0; w < 32; w++) {
        const int q = (w < 16 ? b[2 + w] : b[2 + w - 16] >> 4) & 0x0F;
        y[w] = (float)(q - 8) * d;
    }
}

static void jdq_block_q5_0(const uint8_t *b, float *y) {
    const float d = jdq_half_at(b);
    const uint32_t fifth = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) | ((uint32_t)b[5] << 24);
    for (int w = 0; w < 32; w++) {
        const int nib = (w < 16 ? b[6 + w] : b[6 + w - 16] >> 4) & 0x0F;
        const int q = nib | (int)(((fifth >> w) & 1u) << 4);
        y[w] = (float)(q - 16) * d;
    }
}

static void jdq_block_q8_0(const uint8_t *b, float *y) {
    const float d = jdq_half_at(b);
    for (int w = 0; w < 32; w++) y[w] = (float)(int8_t)b[2 + w] * d;
}

static void jdq_block_q4_k(const uint8_t *b, float *y) {
    const float d = jdq_half_at(b), dmin = jdq_half_at(b + 2);
    const uint8_t *codes = b + 16;
    for (int j = 0; j < 8; j++) {
        int s, m;
        jdq_q4k_scale_min(b + 4, j, &s, &m);
        const float ds = d * (float)s, dm = dmin * (float)m;
        const uint8_t *c = codes + 32 * (j >> 1);
        const int shift = 4 * (j & 1);
        float *out = y + 32 * j;
        for (int l = 0; l < 32; l++) out[l] = ds * (float)((c[l] >> shift) & 0x0F) - dm;
    }
}

static void jdq_block_q6_k(const uint8_t *b, float *y) {
    const float d = jdq_half_at(b + 208);
    for (int half = 0; half < 2; half++) {
        const uint8_t *lo = b + 64 * half, *hi = b + 128 + 32 * half;
        const int8_t *sc = (const int8_t *)(b + 192 + 8 * half);
        for (int u = 0; u < 4; u++) {
            float *out = y + 128 * half + 32 * u;
            const int shift = 4 * (u >> 1);
            for (int l = 0; l < 32; l++) {
                const int q = ((lo[l + 32 * (u & 1)] >> shift) & 0x0F) | (((hi[l] >> (2 * u)) & 3) << 4);
                out[l] = d * (float)sc[l / 16 + 2 * u] * (float)(q - 32);
            }
        }
    }
}

typedef struct {
    int dt;          /* JD_F16, JD_Q4_0, ... */
    int elems;       /* weights per block */
    int bytes;       /* bytes per block */
    void (*decode)(const uint8_t *block, float *out);
} jdq_format;

/* GGUF type ids: F16 1, Q4_0 2, Q5_0 6, Q8_0 8, Q4_K 12, Q6_K 14 */
static const jdq_format JDQ_FORMATS[] = {
    {1, 1, 2, jdq_block_f16},    {2, 32, 18, jdq_block_q4_0},   {6, 32, 22, jdq_block_q5_0},
    {8, 32, 34, jdq_block_q8_0}, {12, 256, 144, jdq_block_q4_k}, {14, 256, 210, jdq_block_q6_k},
};

static inline const jdq_format *jdq_find(int dt) {
    for (unsigned i = 0; i < sizeof JDQ_FORMATS / sizeof JDQ_FORMATS[0]; i++)
        if (JDQ_FORMATS[i].dt == dt) return &JDQ_FORMATS[i];
    return 0;
}

/* Bytes of n weights of type dt (0 for an unknown type); f32 is 4 bytes a weight. */
static inline uint64_t jdq_bytes(int dt, uint64_t n) {
    if (dt == 0) return n * 4;
    const jdq_format *f = jdq_find(dt);
    return f ? (n / (uint64_t)f->elems) * (uint64_t)f->bytes : 0;
}

/* Decode n weights (a whole number of blocks) of type dt into out; -1 for an unknown type. */
static inline int jdq_decode(const uint8_t *src, float *out, uint64_t n, int dt) {
    const jdq_format *f = jdq_find(dt);
    if (!f) return -1;
    for (uint64_t b = 0; b < n / (uint64_t)f->elems; b++) f->decode(src + b * f->bytes, out + b * f->elems);
    return 0;
}
#endif

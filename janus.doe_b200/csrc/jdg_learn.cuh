// jdg_learn.cuh — Hebbian --learn on the device (janusdoe.c:3089-3147, 3416-3447): after a
// token's forward, the prophecy-debt signal of the actual next token, and one "notorch" step
// (Oja-style update of 4 rotating rank lanes toward the captured final hidden x and FFN
// output dy, RMS cap, quarantine) on every LoRA expert elected in that token.  The host
// walks the elected experts in the reference's order and draws the noise from the reference's
// RNG stream, so every update is independent on the device: one CTA each.
#pragma once
#include "jdg_kernels.cuh"

namespace jdg {

constexpr int kLearnLanes = 4;  // NOTORCH_RANK (janusdoe.c:133)

// x and dy RMS-normalised with f64 sums (janusdoe.c:3274-3278, 3311-3315): one CTA
static __global__ __launch_bounds__(1024) void k_learn_capture(const float *xb, const float *dyraw, int D,
                                                               float *x_out, float *dy_out) {
    __shared__ double red[2][32];
    double sx = 0, sd = 0;
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        sx += (double)xb[i] * xb[i];
        sd += (double)dyraw[i] * dyraw[i];
    }
    for (int o = 16; o; o >>= 1) {
        sx += __shfl_xor_sync(JDG_FULL, sx, o);
        sd += __shfl_xor_sync(JDG_FULL, sd, o);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (lane == 0) {
        red[0][warp] = sx;
        red[1][warp] = sd;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double a = 0, b = 0;
        for (int w = 0; w < nw; w++) {
            a += red[0][w];
            b += red[1][w];
        }
        red[0][0] = a;
        red[1][0] = b;
    }
    __syncthreads();
    const float ix = 1.0f / (sqrtf((float)(red[0][0] / D)) + 1e-8f);
    const float id = 1.0f / (sqrtf((float)(red[1][0] / D)) + 1e-8f);
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        x_out[i] = __fmul_rn(xb[i], ix);
        dy_out[i] = __fmul_rn(dyraw[i], id);
    }
}

// signal of the next token (janusdoe.c:3091-3096, 3432-3436): debt pd = diff / (diff + 1)
// with diff = max logit - logit[next]; pd > 0.3 punishes (-pd), else (1 - pd) * 0.1 rewards
static __global__ __launch_bounds__(1024) void k_learn_signal(const float *lg, int V, const int *next, float *sig) {
    __shared__ float red[32];
    float m = -INFINITY;
    for (int i = threadIdx.x; i < V; i += blockDim.x) m = fmaxf(m, lg[i]);
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float mx = red[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) mx = fmaxf(mx, red[w]);
        const int n = *next;
        float s = 0.f;
        if (n >= 0 && n < V) {
            const float diff = mx - lg[n];
            const float pd = diff > 0.f ? diff / (diff + 1.0f) : 0.f;
            s = pd > 0.3f ? -pd : __fmul_rn(1.0f - pd, 0.1f);
        }
        *sig = s;
    }
}

struct LearnUpd {
    int l, e, base;
    float noise[kLearnLanes];
};
struct LearnArgs {
    const LearnUpd *upd;
    float *const *A;   // per layer [16][D][R]
    float *const *B;   // per layer [16][R][D]
    int *const *alive; // per layer [16]
    const float *x, *dy;
    int D, R, nr;
    float lr;          // lr_base * clamped signal
    int *dead;         // [M]
};

// one notorch step + quarantine per CTA (janusdoe.c:3102-3144)
static __global__ __launch_bounds__(256) void k_learn_update(LearnArgs a) {
    __shared__ float u[kLearnLanes];
    __shared__ double dred[2][8];
    __shared__ float fmax_s[8];
    __shared__ int bad_s;
    const LearnUpd up = a.upd[blockIdx.x];
    const int D = a.D, R = a.R, n = D * R, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float *A = a.A[up.l] + (size_t)up.e * D * R, *B = a.B[up.l] + (size_t)up.e * R * D;
    if (tid == 0) bad_s = 0;
    // u_j = clamp(B[r_j] . dy + 0.01 * noise_j, -1, 1) for the rotating lanes r_j
    for (int j = warp; j < a.nr; j += 8) {
        const int r = (up.base + j) % R;
        float s = 0.f;
        for (int i = lane; i < D; i += 32) s = fmaf(B[(size_t)r * D + i], a.dy[i], s);
        s = warp_sum(s);
        if (lane == 0) {
            s = __fadd_rn(s, __fmul_rn(up.noise[j], 0.01f));
            u[j] = fminf(1.0f, fmaxf(-1.0f, s));
        }
    }
    __syncthreads();
    for (int j = 0; j < a.nr; j++) {
        const int r = (up.base + j) % R;
        const float ur = u[j], g = __fmul_rn(a.lr, ur);
        for (int i = tid; i < D; i += blockDim.x) {
            float *pa = A + (size_t)i * R + r;
            *pa = __fadd_rn(*pa, __fmul_rn(g, __fsub_rn(a.x[i], __fmul_rn(ur, *pa))));
            float *pb = B + (size_t)r * D + i;
            *pb = __fadd_rn(*pb, __fmul_rn(g, __fsub_rn(a.dy[i], __fmul_rn(ur, *pb))));
        }
        __syncthreads();
    }
    // soft RMS cap 0.05 on A and on B (f64 sums)
    auto sums = [&](double &sa, double &sb) {
        sa = 0;
        sb = 0;
        for (int i = tid; i < n; i += blockDim.x) {
            sa += (double)A[i] * A[i];
            sb += (double)B[i] * B[i];
        }
        for (int o = 16; o; o >>= 1) {
            sa += __shfl_xor_sync(JDG_FULL, sa, o);
            sb += __shfl_xor_sync(JDG_FULL, sb, o);
        }
        __syncthreads();
        if (lane == 0) {
            dred[0][warp] = sa;
            dred[1][warp] = sb;
        }
        __syncthreads();
        sa = 0;
        sb = 0;
        for (int w = 0; w < 8; w++) {
            sa += dred[0][w];
            sb += dred[1][w];
        }
    };
    double sa, sb;
    sums(sa, sb);
    const float cap = 0.05f, ra = (float)sqrt(sa / n), rb = (float)sqrt(sb / n);
    if (ra > cap) {
        const float f = cap / ra;
        for (int i = tid; i < n; i += blockDim.x) A[i] = __fmul_rn(A[i], f);
    }
    if (rb > cap) {
        const float f = cap / rb;
        for (int i = tid; i < n; i += blockDim.x) B[i] = __fmul_rn(B[i], f);
    }
    __syncthreads();
    // quarantine: a non-finite element, |element| > 8, or RMS over A and B above 5
    float mx = 0.f;
    int bad = 0;
    for (int i = tid; i < n; i += blockDim.x) {
        const float va = A[i], vb = B[i];
        if (!isfinite(va) || !isfinite(vb)) bad = 1;
        mx = fmaxf(mx, fmaxf(fabsf(va), fabsf(vb)));
    }
    mx = warp_max(mx);
    if (bad) atomicOr(&bad_s, 1);
    if (lane == 0) fmax_s[warp] = mx;
    sums(sa, sb);
    if (tid == 0) {
        float m = 0.f;
        for (int w = 0; w < 8; w++) m = fmaxf(m, fmax_s[w]);
        const bool dead = bad_s || m > 8.0f || sqrt((sa + sb) / (2.0 * n)) > 5.0;
        a.dead[blockIdx.x] = dead ? 1 : 0;
        if (dead) a.alive[up.l][up.e] = 0;
    }
}

}  // namespace jdg

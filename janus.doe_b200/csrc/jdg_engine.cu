// jdg_engine.cu — the C ABI of the B200 decode engine (include/jdgpu.h): contexts, weight
// upload, per-sequence state, the decode step as a sequence of sm_100a kernels captured in
// a CUDA graph per batch size, and the device-resident decode loop.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/jdgpu.h"
#include "jdg_engine.h"
#include "jdg_kernels.cuh"
#include "jdg_b1.cuh"
#include "jdg_b1p.cuh"
#include "jdg_tc32.cuh"

using namespace jdg;

struct jdg_ctx {
    int device;
    char err[1024];
};

static thread_local char g_tls_err[1024];

void jdg_set_err(jdg_ctx *c, const char *fmt, ...) {
    char *dst = c ? c->err : g_tls_err;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(dst, 1024, fmt, ap);
    va_end(ap);
}

#define CK(call)                                                                                          \
    do {                                                                                                  \
        cudaError_t _e = (call);                                                                          \
        if (_e != cudaSuccess) {                                                                          \
            jdg_set_err(E_CTX, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(_e), __FILE__, __LINE__); \
            return JD_ECUDA;                                                                              \
        }                                                                                                 \
    } while (0)

// ------------------------------------------------------------------------------------
extern "C" int jdg_device_count(int *n) {
    if (!n) return JD_EINVAL;
    cudaError_t e = cudaGetDeviceCount(n);
    if (e != cudaSuccess) {
        *n = 0;
        return JD_ECUDA;
    }
    return JD_OK;
}

extern "C" int jdg_open(int device, jdg_ctx **out) {
    if (!out) return JD_EINVAL;
    *out = nullptr;
    jdg_ctx *c = (jdg_ctx *)calloc(1, sizeof(jdg_ctx));
    if (!c) return JD_ENOMEM;
    c->device = device;
#define E_CTX c
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        snprintf(g_tls_err, sizeof(g_tls_err), "no CUDA device %d (count %d)", device, n);
        free(c);
        return JD_ECUDA;
    }
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) {
        snprintf(g_tls_err, sizeof(g_tls_err), "cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
        free(c);
        return JD_ECUDA;
    }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) == cudaSuccess && prop.major < 10) {
        snprintf(g_tls_err, sizeof(g_tls_err), "device %d is sm_%d%d; this library is built for sm_100a", device,
                 prop.major, prop.minor);
        free(c);
        return JD_EUNSUPPORTED;
    }
#undef E_CTX
    *out = c;
    return JD_OK;
}

extern "C" void jdg_close(jdg_ctx *c) { free(c); }

extern "C" const char *jdg_last_error(jdg_ctx *c) { return c ? c->err : g_tls_err; }

int jdg_ctx_device(jdg_ctx *c) { return c->device; }

// ------------------------------------------------------------------------------------
// Device arena: one allocation, 256-byte aligned sub-buffers.
struct Arena {
    std::vector<std::pair<size_t *, size_t>> req;
};

static size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

#define E_CTX (e->ctx)

static int dev_alloc(jdg_engine *e, void **p, size_t bytes) {
    cudaError_t r = cudaMalloc(p, bytes ? bytes : 256);
    if (r != cudaSuccess) {
        jdg_set_err(e->ctx, "cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(r));
        return JD_ENOMEM;
    }
    e->allocs.push_back(*p);
    return JD_OK;
}
#define DALLOC(ptr, bytes)                                              \
    do {                                                                \
        int _r = dev_alloc(e, (void **)&(ptr), (size_t)(bytes));        \
        if (_r != JD_OK) return _r;                                     \
    } while (0)

static int h2d(jdg_engine *e, void *dst, const void *src, size_t bytes) {
    CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, e->st));
    return JD_OK;
}

// common state buffers: tokens, positions, prompts, history, RNG, EMA, trace, election
int jdg_alloc_state(jdg_engine *e) {
    const int B = e->B_max, L = e->L;
    DALLOC(e->tok, B * 4);
    DALLOC(e->pos, B * 4);
    DALLOC(e->plen, B * 4);
    DALLOC(e->next_out, B * 4);
    DALLOC(e->hist_n, B * 4);
    DALLOC(e->rng, B * 8);
    e->Pmax = e->max_seq;
    e->Hmax = e->max_seq;
    DALLOC(e->prompt, (size_t)B * e->Pmax * 4);
    DALLOC(e->hist, (size_t)B * e->Hmax * 4);
    DALLOC(e->consensus, (size_t)B * L * 4);
    DALLOC(e->kcnt, B * 4);
    DALLOC(e->sel, (size_t)B * kMaxE * 4);
    DALLOC(e->selw, (size_t)B * kMaxE * 4);
    DALLOC(e->rcnt, kMaxE * 4);
    DALLOC(e->ridx, (size_t)kMaxE * B * 4);
    DALLOC(e->pairrow, (size_t)B * kMaxE * 4);
    DALLOC(e->tr_k, (size_t)B * L * 4);
    DALLOC(e->tr_ema, (size_t)B * L * 4);
    DALLOC(e->tr_sel, (size_t)B * L * kMaxE * 4);
    DALLOC(e->tr_w, (size_t)B * L * kMaxE * 4);
    DALLOC(e->err, 4);
    CK(cudaMemsetAsync(e->err, 0, 4, e->st));
    DALLOC(e->stats, 4 * 8);
    CK(cudaMemsetAsync(e->stats, 0, 4 * 8, e->st));
    if (cudaHostAlloc((void **)&e->pin_tok, (size_t)B * 12 + 64, cudaHostAllocDefault) != cudaSuccess) {
        jdg_set_err(e->ctx, "cudaHostAlloc failed");
        return JD_ENOMEM;
    }
    e->pin_pos = e->pin_tok + B;
    e->pin_next = e->pin_pos + B;
    e->pin_err = e->pin_next + B;  // in the 64 spare bytes
    DALLOC(e->tickets, 1024 * 4);
    CK(cudaMemsetAsync(e->tickets, 0, 1024 * 4, e->st));
    CK(cudaMemsetAsync(e->tok, 0, B * 4, e->st));
    CK(cudaMemsetAsync(e->pos, 0, B * 4, e->st));
    CK(cudaMemsetAsync(e->plen, 0, B * 4, e->st));
    CK(cudaMemsetAsync(e->hist_n, 0, B * 4, e->st));
    CK(cudaMemsetAsync(e->rng, 0, B * 8, e->st));
    CK(cudaMemsetAsync(e->tr_k, 0, (size_t)B * L * 4, e->st));
    return JD_OK;
}

int jdg_engine_create(jdg_ctx *ctx, int kind, jdg_engine **out);
static int engine_new(jdg_ctx *ctx, int kind, jdg_engine **out) { return jdg_engine_create(ctx, kind, out); }
int jdg_engine_create(jdg_ctx *ctx, int kind, jdg_engine **out) {
    jdg_engine *e = new (std::nothrow) jdg_engine();
    if (!e) return JD_ENOMEM;
    e->ctx = ctx;
    e->kind = kind;
    e->temp = 0.f;
    e->top_k = 0;
    cudaError_t r = cudaSetDevice(ctx->device);
    if (r == cudaSuccess) r = cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking);
    if (r == cudaSuccess) r = cudaEventCreate(&e->ev0);
    if (r == cudaSuccess) r = cudaEventCreate(&e->ev1);
    if (r != cudaSuccess) {
        jdg_set_err(ctx, "stream/event create: %s", cudaGetErrorString(r));
        delete e;
        return JD_ECUDA;
    }
    *out = e;
    return JD_OK;
}

// ------------------------------------------------------------------------------------
// Own-model upload.  Device layout per layer: wqkv = [wq; wk; wv] (rows), wo, w_vote,
// and per alive expert gu = interleaved rows (gate_i, up_i) [2H][D] and down [D][H].
extern "C" int jdg_own_upload(jdg_ctx *ctx, const jd_model *m, int max_batch, jdg_engine **out) {
    if (!ctx || !m || !out || !m->tok_emb || max_batch < 1 || max_batch > 4096) {
        if (ctx) jdg_set_err(ctx, "jdg_own_upload: bad arguments");
        return JD_EINVAL;
    }
    const jd_config &c = m->c;
    if (c.depth < 1 || c.depth > JD_MAX_LAYERS || c.n_kv_heads < 1 || c.n_heads % c.n_kv_heads ||
        (c.head_dim != 64 && c.head_dim != 128) || c.n_heads / c.n_kv_heads > kMaxHG || c.dim % 16 ||
        c.hidden_dim % 16 || (c.n_heads * c.head_dim) % 16 || c.seq_len < 1) {
        jdg_set_err(ctx, "jdg_own_upload: unsupported config (dim %d heads %d/%d hd %d hidden %d)", c.dim, c.n_heads,
                    c.n_kv_heads, c.head_dim, c.hidden_dim);
        return JD_EUNSUPPORTED;
    }
    jdg_engine *e = nullptr;
    int rc = engine_new(ctx, 0, &e);
    if (rc != JD_OK) return rc;
    rc = jdg_own_upload_impl(e, m, max_batch);
    if (rc != JD_OK) {
        jdg_engine_free(e);
        return rc;
    }
    *out = e;
    return JD_OK;
}

static bool b1p_usable(jdg_engine *e);
static int tc_build(jdg_engine *e, const jd_model *m);

int jdg_own_upload_impl(jdg_engine *e, const jd_model *m, int max_batch) {
    const jd_config &c = m->c;
    e->B_max = max_batch;
    e->L = (c.active_depth > 0 && c.active_depth <= c.depth) ? c.active_depth : c.depth;
    e->D = c.dim;
    e->Hh = c.n_heads;
    e->KVH = c.n_kv_heads;
    e->HD = c.head_dim;
    e->hidden = c.hidden_dim;
    e->V = c.vocab_size;
    e->ldl = c.vocab_size;
    e->max_seq = c.seq_len;
    e->qd = c.n_heads * c.head_dim;
    e->kd = c.n_kv_heads * c.head_dim;
    e->qkvd = e->qd + 2 * e->kd;
    e->eps = c.norm_eps;
    e->clamp = c.attn_clamp;
    if (jdg_attn_setup(e) != JD_OK) return JD_ECUDA;
    const int D = e->D, H = e->hidden, L = e->L, V = e->V;
    // weight arena
    size_t bytes = al256((size_t)V * D * 4) * 2 + al256(D * 4);
    int kmax = 0;
    for (int l = 0; l < L; l++) {
        const jd_layer &ly = m->layers[l];
        bytes += al256(D * 4) * 2 + al256((size_t)e->qkvd * D * 4) + al256((size_t)D * e->qd * 4) +
                 al256((size_t)kMaxE * D * 4);
        int na = 0;
        for (int x = 0; x < kMaxE; x++)
            if (ly.alive[x]) {
                if (!ly.w_gate[x] || !ly.w_up[x] || !ly.w_down[x]) {
                    jdg_set_err(e->ctx, "layer %d expert %d alive without weights", l, x);
                    return JD_EINVAL;
                }
                bytes += al256((size_t)2 * H * D * 4) + al256((size_t)D * H * 4);
                na++;
            }
        if (na > kmax) kmax = na;
        e->n_alive[l] = na;
    }
    e->kmax = kmax < 1 ? 1 : kmax;
    DALLOC(e->arena, bytes);
    char *p = (char *)e->arena;
    auto take = [&](size_t b) {
        char *r = p;
        p += al256(b);
        return r;
    };
    std::vector<float> tmp;
    e->tok_emb = (float *)take((size_t)V * D * 4);
    e->output = (float *)take((size_t)V * D * 4);
    e->output_norm = (float *)take(D * 4);
    CK(cudaMemcpy(e->tok_emb, m->tok_emb, (size_t)V * D * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(e->output, m->output, (size_t)V * D * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(e->output_norm, m->output_norm, D * 4, cudaMemcpyHostToDevice));
    std::vector<float *> gu((size_t)L * kMaxE, nullptr), dn((size_t)L * kMaxE, nullptr);
    std::vector<int> alive((size_t)L * kMaxE, 0);
    for (int l = 0; l < L; l++) {
        const jd_layer &ly = m->layers[l];
        LayerDev &ld = e->layers[l];
        ld.attn_norm = (float *)take(D * 4);
        ld.ffn_norm = (float *)take(D * 4);
        ld.wqkv = (float *)take((size_t)e->qkvd * D * 4);
        ld.wo = (float *)take((size_t)D * e->qd * 4);
        ld.w_vote = (float *)take((size_t)kMaxE * D * 4);
        ld.temperature = ly.temperature;
        CK(cudaMemcpy(ld.attn_norm, ly.attn_norm, D * 4, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(ld.ffn_norm, ly.ffn_norm, D * 4, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(ld.wqkv, ly.wq, (size_t)e->qd * D * 4, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(ld.wqkv + (size_t)e->qd * D, ly.wk, (size_t)e->kd * D * 4, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(ld.wqkv + (size_t)(e->qd + e->kd) * D, ly.wv, (size_t)e->kd * D * 4, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(ld.wo, ly.wo, (size_t)D * e->qd * 4, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(ld.w_vote, ly.w_vote, (size_t)kMaxE * D * 4, cudaMemcpyHostToDevice));
        for (int x = 0; x < kMaxE; x++) {
            if (!ly.alive[x]) continue;
            float *g = (float *)take((size_t)2 * H * D * 4);
            float *d = (float *)take((size_t)D * H * 4);
            tmp.resize((size_t)2 * H * D);
            for (int i = 0; i < H; i++) {
                memcpy(&tmp[(size_t)(2 * i) * D], ly.w_gate[x] + (size_t)i * D, D * 4);
                memcpy(&tmp[(size_t)(2 * i + 1) * D], ly.w_up[x] + (size_t)i * D, D * 4);
            }
            CK(cudaMemcpy(g, tmp.data(), (size_t)2 * H * D * 4, cudaMemcpyHostToDevice));
            CK(cudaMemcpy(d, ly.w_down[x], (size_t)D * H * 4, cudaMemcpyHostToDevice));
            gu[(size_t)l * kMaxE + x] = g;
            dn[(size_t)l * kMaxE + x] = d;
            alive[(size_t)l * kMaxE + x] = 1;
        }
        e->layer_consensus[l] = ly.consensus;
    }
    DALLOC(e->gu_tab, (size_t)L * kMaxE * sizeof(float *));
    DALLOC(e->dn_tab, (size_t)L * kMaxE * sizeof(float *));
    DALLOC(e->alive_dev, (size_t)L * kMaxE * 4);
    CK(cudaMemcpy(e->gu_tab, gu.data(), gu.size() * sizeof(float *), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(e->dn_tab, dn.data(), dn.size() * sizeof(float *), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(e->alive_dev, alive.data(), alive.size() * 4, cudaMemcpyHostToDevice));
    {   // per-layer parameter blocks of the persistent batch-1 step: header (weight pointers,
        // alive mask, temperature), attn_norm, ffn_norm, factored vote rows wvn[r][e]
        const size_t stride = b1p_par_stride(D);
        std::vector<char> blk((size_t)L * stride, 0);
        for (int l = 0; l < L; l++) {
            const jd_layer &ly = m->layers[l];
            char *b = blk.data() + (size_t)l * stride;
            B1PLayer q;
            memset(&q, 0, sizeof q);
            q.wqkv = e->layers[l].wqkv;
            q.wo = e->layers[l].wo;
            q.temperature = e->layers[l].temperature;
            for (int x = 0; x < kMaxE; x++) {
                q.gu[x] = gu[(size_t)l * kMaxE + x];
                q.dn[x] = dn[(size_t)l * kMaxE + x];
                if (alive[(size_t)l * kMaxE + x]) q.alive |= 1u << x;
            }
            memcpy(b, &q, sizeof q);
            float *an = reinterpret_cast<float *>(b + kPParHdr), *fn = an + D, *wvn = fn + D;
            memcpy(an, ly.attn_norm, (size_t)D * 4);
            memcpy(fn, ly.ffn_norm, (size_t)D * 4);
            for (int r = 0; r < D; r++)
                for (int x = 0; x < kMaxE; x++)
                    wvn[r * kMaxE + x] = (q.alive >> x & 1u) ? ly.w_vote[(size_t)x * D + r] * ly.ffn_norm[r] : 0.f;
        }
        DALLOC(e->b1p_layers, blk.size());
        CK(cudaMemcpy(e->b1p_layers, blk.data(), blk.size(), cudaMemcpyHostToDevice));
    }
    // RoPE cache as alloc_run builds it (janusdoe.c:866-873)
    const int half = e->HD / 2;
    std::vector<float> cs((size_t)e->max_seq * half), sn((size_t)e->max_seq * half);
    for (int pp = 0; pp < e->max_seq; pp++)
        for (int i = 0; i < half; i++) {
            float freq = 1.0f / powf(c.rope_theta, (float)(2 * i) / (float)c.head_dim);
            float ang = (float)pp * freq;
            cs[(size_t)pp * half + i] = cosf(ang);
            sn[(size_t)pp * half + i] = sinf(ang);
        }
    DALLOC(e->rope_cos, cs.size() * 4);
    DALLOC(e->rope_sin, sn.size() * 4);
    CK(cudaMemcpy(e->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(e->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
    e->rope_norm = 0;
    // activations
    const int B = max_batch;
    DALLOC(e->x, (size_t)B * D * 4);
    DALLOC(e->xb, (size_t)B * D * 4);
    DALLOC(e->qkv, (size_t)B * e->qkvd * 4);
    DALLOC(e->att, (size_t)B * e->qd * 4);
    size_t part_a = (size_t)B * e->Hh * e->nchunk * (e->HD + 2);
    size_t part_b = (size_t)e->Hh * (e->max_seq / kB1Chunk + 1) * (e->HD + 2);
    size_t part_c = (size_t)e->Hh * (e->max_seq / kPChunk + 1) * (e->HD + 2);
    part_b = part_b > part_c ? part_b : part_c;
    DALLOC(e->part, (part_a > part_b ? part_a : part_b) * 4);
    DALLOC(e->amax_v, ((size_t)V / 4 + 2) * 4);
    DALLOC(e->amax_i, ((size_t)V / 4 + 2) * 4);
    DALLOC(e->vpart, ((size_t)D / 4 + 2 > 1024 ? (size_t)D / 4 + 2 : 1024) * 17 * 4);
    DALLOC(e->sel_gu, kMaxE * sizeof(float *));
    DALLOC(e->ema_new, 4);
    DALLOC(e->x2, (size_t)D * 4);
    DALLOC(e->sel_dn, kMaxE * sizeof(float *));
    DALLOC(e->ffn_inv, 4);
    {
        const char *g = getenv("JDG_GENERIC");
        e->force_generic = g && g[0] == '1';
        // batch-1 own-model path: the persistent one-kernel step ("step") or the kernel chain
        const char *c = getenv("JDG_B1");
        e->force_chain = !(c && !strcmp(c, "step"));
    }
    e->b1_ok = D % 128 == 0 && H % 128 == 0 && D / 128 <= 8 && H / 128 <= 12 && e->qd == D && D <= 1024 &&
               (e->HD == 64 || e->HD == 128) && D / 4 + 64 <= 1024 && e->max_seq <= 1024;
    DALLOC(e->hbuf, (size_t)B * kMaxE * 2 * H * 4);  // batched tensor-core step: [slot][B][2H]
    DALLOC(e->ybuf, (size_t)B * kMaxE * D * 4);
    CK(cudaMemset(e->ybuf, 0, (size_t)B * kMaxE * D * 4));
    CK(cudaMemset(e->hbuf, 0, (size_t)B * kMaxE * 2 * H * 4));
    DALLOC(e->logits, (size_t)B * V * 4);
    // KV cache [B][L][S][kd]
    e->kv_bstride = (long)L * e->max_seq * e->kd;
    DALLOC(e->kc, (size_t)B * e->kv_bstride * 4);
    DALLOC(e->vc, (size_t)B * e->kv_bstride * 4);
    int rc = jdg_alloc_state(e);
    if (rc != JD_OK) return rc;
    rc = jdg_reset(e, -1);
    if (rc != JD_OK) return rc;
    CK(cudaStreamSynchronize(e->st));
    b1p_usable(e);  // decided here, outside any stream capture
    rc = tc_build(e, m);
    if (rc != JD_OK) return rc;
    return JD_OK;
}

// ------------------------------------------------------------------------------------
// Tensor-core blocks of every own-model matrix the batched step multiplies (TF32 hi/lo in the
// MMA layout, jdg_tc32.cuh), built on the device from the uploaded f32 weights.
static size_t tc_blocks_bytes(int N, int K) { return (size_t)((N + kTcRows - 1) / kTcRows) * (K / kTcK) * 2 * kTcBlk; }

static int tc_blocks(jdg_engine *e, const float *W, int N, int K, uint8_t **out) {
    DALLOC(*out, tc_blocks_bytes(N, K));
    k_tc_wprep<<<1184, 256, 0, e->st>>>(W, N, K, *out);
    return JD_OK;
}

static int tc_table(jdg_engine *e, const uint8_t *const *ptrs, int n, const uint8_t ***out) {
    DALLOC(*out, (size_t)n * sizeof(void *));
    CK(cudaMemcpy((void *)*out, ptrs, (size_t)n * sizeof(void *), cudaMemcpyHostToDevice));
    return JD_OK;
}

static int tc_build(jdg_engine *e, const jd_model *m) {
    const char *g = getenv("JDG_SIMT_GEMM");
    if ((g && g[0] == '1') || e->D % kTcK || e->hidden % kTcK || e->qd % kTcK) return JD_OK;
    const int D = e->D, H = e->hidden, L = e->L;
    {  // the activation prep indexes segments x token tiles x 128 x K/4 in 32 bits
        const uint64_t rows = (uint64_t)std::max(e->B_max, e->max_seq) + kTcTok;
        const uint64_t kq = (uint64_t)std::max(std::max(D, H), e->qd) / 4;
        if ((uint64_t)kMaxE * rows * kq >= (1ull << 32)) return JD_OK;
    }
    std::vector<const float *> gu_h((size_t)L * kMaxE), dn_h((size_t)L * kMaxE);
    CK(cudaMemcpy(gu_h.data(), e->gu_tab, gu_h.size() * sizeof(void *), cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(dn_h.data(), e->dn_tab, dn_h.size() * sizeof(void *), cudaMemcpyDeviceToHost));
    for (int l = 0; l < L; l++) {
        LayerDev &ly = e->layers[l];
        int rc = tc_blocks(e, ly.wqkv, e->qkvd, D, &ly.tc_wqkv);
        if (rc == JD_OK) rc = tc_blocks(e, ly.wo, D, e->qd, &ly.tc_wo);
        if (rc != JD_OK) return rc;
        const uint8_t *gt[kMaxE] = {nullptr}, *dt[kMaxE] = {nullptr};
        for (int x = 0; x < kMaxE; x++) {
            if (!gu_h[(size_t)l * kMaxE + x]) continue;
            uint8_t *b1 = nullptr, *b2 = nullptr;
            rc = tc_blocks(e, gu_h[(size_t)l * kMaxE + x], 2 * H, D, &b1);
            if (rc == JD_OK) rc = tc_blocks(e, dn_h[(size_t)l * kMaxE + x], D, H, &b2);
            if (rc != JD_OK) return rc;
            gt[x] = b1;
            dt[x] = b2;
        }
        const uint8_t *one[1] = {ly.tc_wqkv}, *two[1] = {ly.tc_wo};
        int rc2 = tc_table(e, gt, kMaxE, &ly.tc_gu);
        if (rc2 == JD_OK) rc2 = tc_table(e, dt, kMaxE, &ly.tc_dn);
        if (rc2 == JD_OK) rc2 = tc_table(e, one, 1, &ly.tc_wqkv_tab);
        if (rc2 == JD_OK) rc2 = tc_table(e, two, 1, &ly.tc_wo_tab);
        if (rc2 != JD_OK) return rc2;
    }
    int rc = tc_blocks(e, e->output, e->V, D, &e->tc_out);
    if (rc != JD_OK) return rc;
    const uint8_t *ot[1] = {e->tc_out};
    rc = tc_table(e, ot, 1, &e->tc_out_tab);
    if (rc != JD_OK) return rc;
    // activation blocks for up to max(batch, context) rows in 16 segments, the widest K
    const int rows = std::max(e->B_max, e->max_seq), kmax = std::max(D, H);
    const int tt = (rows + kTcTok - 1) / kTcTok;
    e->tc_xt_bytes = (size_t)kMaxE * tt * (kmax / kTcK) * 2 * kTcBlk;
    DALLOC(e->tc_xt, e->tc_xt_bytes);
    DALLOC(e->tc_part, (size_t)64 << 20);
    CK(cudaFuncSetAttribute(k_tc32_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem));
    CK(cudaStreamSynchronize(e->st));
    e->tc_ok = 1;
    return JD_OK;
}

// C = X.W^T on the tensor cores: X rows from `X` (segment s at X + s*x_seg, rows idx[s*ldi+j]
// when idx is given, counts cnt[s] or M), W as per-segment block tables `wt` (n_rows x K).
static void launch_tc(jdg_engine *e, const uint8_t *const *wt, int nseg, const float *X, long x_seg, int ldx,
                      const int *idx, int ldi, const int *cnt, int M, int max_rows, int n_rows, int K, float *C,
                      int ldc, long c_seg, int epi, float alpha, int x_glu = 0, int x_ready = 0,
                      SplitPart *fuse = nullptr) {
    const int ttiles = (max_rows + kTcTok - 1) / kTcTok, nkc = K / kTcK;
    TcPrep p = {};
    p.X = X; p.x_seg = x_seg; p.ldx = ldx; p.K = K; p.idx = idx; p.ldi = ldi; p.cnt = cnt; p.M = M;
    p.nseg = nseg; p.ttiles = ttiles; p.glu = x_glu; p.out = e->tc_xt;
    if (!x_ready) {  // else the producing kernel wrote the blocks (k_tc_norm_prep, k_tc_combine_prep)
        k_tc_xprep<<<1184, 256, 0, e->st>>>(p);
        e->launches++;
    }
    const int rtiles = (n_rows + kTcRows - 1) / kTcRows;
    // split K until about one CTA per SM (every split keeps at least one chunk)
    int ks = 1;
    const int tiles = rtiles * ttiles * nseg;
    if (nseg == 1)
        while (ks < kTcMaxSplit && tiles * (ks + 1) <= 148 && nkc / (ks + 1) >= 2) ks++;
    const int per = (nkc + ks - 1) / ks;
    ks = (nkc + per - 1) / per;
    TcArgs a = {};
    a.wt = wt; a.xt = e->tc_xt; a.cnt = cnt; a.M = M; a.n_rows = n_rows; a.nkc = nkc; a.ttiles = ttiles;
    a.C = C; a.ldc = ldc; a.c_seg = c_seg; a.epi = epi; a.alpha = alpha; a.ksplit = ks; a.part = e->tc_part;
    a.err = e->err;
    a.tl = e->timeline;  // debug wait profile: 0 q/k/v, 1 Wo, 2 gate/up, 3 down, 4 LM head
    a.tl_type = nseg > 1 ? (x_glu ? 3 : 2) : epi == EPI_ADD ? 1 : n_rows == e->V ? 4 : 0;
    k_tc32_gemm<<<dim3(rtiles, ttiles, nseg * ks), kTcThreads, kTcSmem, e->st>>>(a);
    e->launches++;
    if (fuse) *fuse = SplitPart{nullptr, 1, rtiles};
    if (ks > 1 && fuse && nseg == 1) {  // the consumer sums the partials (split_sum)
        *fuse = SplitPart{e->tc_part, ks, rtiles};
    } else if (ks > 1) {
        const long items = (long)nseg * ttiles * rtiles * kTcTok * (kTcRows / 4);
        k_tc_reduce<<<(int)std::min<long>((items + 255) / 256, 148 * 8), 256, 0, e->st>>>(a, rtiles, nseg);
        e->launches++;
    }
}

static int pick_bm(int B) { return B <= 16 ? 16 : B <= 32 ? 32 : 64; }

template <int EPI>
static void launch_sgemm(jdg_engine *e, const SgemmArgs &a, int B, int nseg) {
    dim3 grid((a.N + 127) / 128, (B + pick_bm(B) - 1) / pick_bm(B), nseg);
    switch (pick_bm(B)) {
    case 16: k_sgemm<16, EPI><<<grid, 256, 0, e->st>>>(a); break;
    case 32: k_sgemm<32, EPI><<<grid, 256, 0, e->st>>>(a); break;
    default: k_sgemm<64, EPI><<<grid, 256, 0, e->st>>>(a); break;
    }
    e->launches++;
}

static void launch_gemv1(jdg_engine *e, int epi, const float *W, int N, int K, const float *X, const float *norm_w,
                         int prenorm, float *Y) {
    GemvArgs a = {};
    a.W = W;
    a.N = N;
    a.K = K;
    a.X = X;
    a.ldx = K;
    a.norm_w = norm_w;
    a.eps = e->eps;
    a.prenorm = prenorm;
    a.Y = Y;
    a.ldy = N;
    int grid = (N + 3) / 4;
    size_t sm = (size_t)K * 4;
    if (epi == EPI_ADD) k_gemv_f32<1, 1, EPI_ADD><<<grid, 128, sm, e->st>>>(a);
    else k_gemv_f32<1, 1, EPI_STORE><<<grid, 128, sm, e->st>>>(a);
    e->launches++;
}

// tc_prep: the merge writes the Wo product's activation blocks instead of att
static void launch_attention(jdg_engine *e, int l, int B, float scale, float bias, bool tc_prep = false) {
    AttnArgs a = {};
    a.qkv = e->qkv;
    a.ld = e->qkvd;
    a.kc = e->kc + (size_t)l * e->max_seq * e->kd;
    a.vc = e->vc + (size_t)l * e->max_seq * e->kd;
    a.bstride = e->kv_bstride;
    a.pos = e->pos;
    a.H = e->Hh;
    a.KVH = e->KVH;
    a.HD = e->HD;
    a.hg = e->Hh / e->KVH;
    a.nchunk = e->nchunk;
    a.scale = scale;
    a.bias = bias;
    a.clamp = e->clamp;
    a.inv_clamp = e->clamp > 0 ? 1.0f / e->clamp : 0.f;
    a.part = e->part;
    int chunk = kAttnChunk;
    if (e->attn_rows) {
        chunk = kAttnRowsChunk;
        dim3 grid((e->max_seq + chunk - 1) / chunk, B);
        const size_t sm = attn_rows_smem(e->Hh, e->HD, e->kd);
        if (e->HD == 64) k_attn_rows<64><<<grid, e->Hh * 32, sm, e->st>>>(a);
        else k_attn_rows<128><<<grid, e->Hh * 32, sm, e->st>>>(a);
    } else {
        dim3 grid((e->max_seq + chunk - 1) / chunk, e->KVH, B);
        if (e->HD == 64) k_attn_partial<64><<<grid, 128, 0, e->st>>>(a);
        else k_attn_partial<128><<<grid, 128, 0, e->st>>>(a);
    }
    if (tc_prep)
        k_tc_combine_prep<<<dim3(e->Hh, B), e->HD, (size_t)2 * e->nchunk * 4, e->st>>>(e->part, e->pos, e->Hh, e->HD,
                                                                                e->nchunk, chunk, e->tc_xt);
    else
        k_attn_combine<<<dim3(e->Hh, B), e->HD, (size_t)2 * e->nchunk * 4, e->st>>>(e->part, e->pos, e->Hh, e->HD,
                                                                             e->nchunk, chunk, e->att, e->qd);
    e->launches += 2;
}

// Pick the attention kernel for this engine's shapes (at upload, outside any capture):
// k_attn_rows when a chunk's key and value rows fit shared memory and the heads fit one CTA.
int jdg_attn_setup(jdg_engine *e) {
    const size_t sm = attn_rows_smem(e->Hh, e->HD, e->kd);
    e->attn_rows = (e->HD == 64 || e->HD == 128) && e->Hh <= 32 && e->Hh % e->KVH == 0 && sm <= 160 * 1024;
    if (e->attn_rows) {
        cudaError_t r = e->HD == 64
                            ? cudaFuncSetAttribute(k_attn_rows<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm)
                            : cudaFuncSetAttribute(k_attn_rows<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (r != cudaSuccess) {
            jdg_set_err(e->ctx, "attention smem attribute: %s", cudaGetErrorString(r));
            return JD_ECUDA;
        }
    }
    // partial buffers are laid out for the smaller chunk
    e->nchunk = (e->max_seq + kAttnRowsChunk - 1) / kAttnRowsChunk;
    return JD_OK;
}

void jdg_launch_rope(jdg_engine *e, int l, int B, SplitPart sp) {
    RopeArgs r = {};
    r.qkv = e->qkv;
    r.ld = e->qkvd;
    r.H = e->Hh;
    r.KVH = e->KVH;
    r.HD = e->HD;
    r.cos_t = e->rope_cos;
    r.sin_t = e->rope_sin;
    r.pair_norm = e->rope_norm;
    r.pos = e->pos;
    r.max_seq = e->max_seq;
    r.kc = e->kc + (size_t)l * e->max_seq * e->kd;
    r.vc = e->vc + (size_t)l * e->max_seq * e->kd;
    r.bstride = e->kv_bstride;
    r.err = e->err;
    r.sp = sp;
    k_rope_kv<<<B, 256, 0, e->st>>>(r);
    e->launches++;
}

void jdg_launch_attention(jdg_engine *e, int l, int B, float scale, float bias) { launch_attention(e, l, B, scale, bias); }

void jdg_launch_pick(jdg_engine *e, int B) {
    PickArgs pa = {};
    pa.logits = e->logits;
    pa.V = e->ldl;
    pa.ldl = e->ldl;
    pa.temp = e->temp;
    pa.top_k = e->top_k;
    pa.tok = e->tok;
    pa.pos = e->pos;
    pa.rng = e->rng;
    pa.plen = e->plen;
    pa.prompt = e->prompt;
    pa.Pmax = e->Pmax;
    pa.hist = e->hist;
    pa.hist_n = e->hist_n;
    pa.Hmax = e->Hmax;
    pa.next_out = e->next_out;
    pa.stats = e->stats;
    k_pick<<<B, 1024, 0, e->st>>>(pa);
    e->launches++;
}

void jdg_launch_pick_tp(jdg_engine *e, int B, const float *v, const int *ix, int world) {
    k_pick_tp<<<(B + 127) / 128, 128, 0, e->st>>>(v, ix, world, B, e->tok, e->pos, e->plen, e->prompt, e->Pmax, e->hist,
                                                  e->hist_n, e->Hmax, e->next_out, e->stats);
}

void jdg_launch_elect(jdg_engine *e, int l, int B, const float *xin, const float *norm_w, const float *w_vote,
                      const int *alive, float temperature, int host, SplitPart sp) {
    ElectArgs a = {};
    a.x = xin;
    a.sp = sp;
    a.x_out = e->x;
    a.norm_w = norm_w;
    a.eps = e->eps;
    a.D = e->D;
    a.host = host;
    a.w_vote = w_vote;
    a.alive = alive;
    a.temperature = temperature;
    a.consensus = e->consensus;
    a.L = e->L;
    a.l = l;
    a.xb = e->xb;
    a.kcnt = e->kcnt;
    a.sel = e->sel;
    a.selw = e->selw;
    a.tr_k = e->tr_k;
    a.tr_sel = e->tr_sel;
    a.tr_w = e->tr_w;
    a.tr_ema = e->tr_ema;
    k_elect<<<B, 256, (size_t)e->D * 4, e->st>>>(a);
    e->launches++;
}


// ------------------------------------------------------------------------------------
// Batch-1 chain (jdg_b1.cuh), every kernel launched with programmatic stream serialization.
template <typename... KArgs, typename... Args>
static void launch_pdl_sm(jdg_engine *e, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = e->st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, args...);
    e->launches++;
}
template <typename... KArgs, typename... Args>
static void launch_pdl(jdg_engine *e, void (*kern)(KArgs...), dim3 grid, dim3 block, Args... args) {
    launch_pdl_sm(e, kern, grid, block, 0, args...);
}

#define NV_SWITCH(n, KERN, ...)                                        \
    switch (n) {                                                       \
    case 2: launch_pdl(e, KERN<2>, __VA_ARGS__); break;                \
    case 4: launch_pdl(e, KERN<4>, __VA_ARGS__); break;                \
    case 6: launch_pdl(e, KERN<6>, __VA_ARGS__); break;                \
    default: launch_pdl(e, KERN<8>, __VA_ARGS__); break;               \
    }
#define NH_SWITCH(n, KERN, ...)                                        \
    switch (n) {                                                       \
    case 3: launch_pdl(e, KERN<3>, __VA_ARGS__); break;                \
    case 4: launch_pdl(e, KERN<4>, __VA_ARGS__); break;                \
    case 6: launch_pdl(e, KERN<6>, __VA_ARGS__); break;                \
    case 8: launch_pdl(e, KERN<8>, __VA_ARGS__); break;                \
    case 9: launch_pdl(e, KERN<9>, __VA_ARGS__); break;                \
    default: launch_pdl(e, KERN<12>, __VA_ARGS__); break;              \
    }

#define WO_SWITCH(n, HDV, ...)                                         \
    switch (n) {                                                       \
    case 2: launch_pdl(e, k_b1_wo<2, HDV>, __VA_ARGS__); break;        \
    case 4: launch_pdl(e, k_b1_wo<4, HDV>, __VA_ARGS__); break;        \
    case 6: launch_pdl(e, k_b1_wo<6, HDV>, __VA_ARGS__); break;        \
    default: launch_pdl(e, k_b1_wo<8, HDV>, __VA_ARGS__); break;       \
    }
static bool b1_shape_ok(jdg_engine *e) {
    int nv = e->D / 128, nh = e->hidden / 128;
    return e->b1_ok && (nv == 2 || nv == 4 || nv == 6 || nv == 8) &&
           (nh == 3 || nh == 4 || nh == 6 || nh == 8 || nh == 9 || nh == 12);
}

static void enqueue_own_step_b1(jdg_engine *e) {
    B1Args a = {};
    a.tok_emb = e->tok_emb;
    a.V = e->V; a.D = e->D; a.H = e->Hh; a.KVH = e->KVH; a.HD = e->HD; a.hidden = e->hidden;
    a.qd = e->qd; a.kd = e->kd; a.qkvd = e->qkvd; a.max_seq = e->max_seq; a.L = e->L;
    a.eps = e->eps; a.scale = 1.0f / sqrtf((float)e->HD); a.clamp = e->clamp;
    a.inv_clamp = e->clamp > 0 ? 1.0f / e->clamp : 0.f;
    a.rope_norm = 0; a.rope_cos = e->rope_cos; a.rope_sin = e->rope_sin;
    a.output = e->output; a.output_norm = e->output_norm;
    a.tok = e->tok; a.pos = e->pos; a.x = e->x; a.xb = e->xb; a.qkv = e->qkv; a.att = e->att; a.part = e->part;
    a.hbuf = e->hbuf; a.ybuf = e->ybuf; a.logits = e->logits; a.kv_bstride = e->kv_bstride;
    a.kcnt = e->kcnt; a.sel = e->sel; a.selw = e->selw; a.consensus = e->consensus;
    a.tickets = e->tickets; a.amax_v = e->amax_v; a.amax_i = e->amax_i; a.vpart = e->vpart; a.ffn_inv = e->ffn_inv;
    a.tok_out = e->tok; a.plen = e->plen; a.prompt = e->prompt; a.hist = e->hist; a.hist_n = e->hist_n;
    a.next_out = e->next_out; a.Pmax = e->Pmax; a.Hmax = e->Hmax; a.err = e->err;
    a.greedy_pick = e->temp <= 0.f;
    a.stats = e->stats;
    a.sel_gu = e->sel_gu;
    a.sel_dn = e->sel_dn;
    a.tl = e->timeline;
    const int nv = e->D / 128, nh = e->hidden / 128;
    const dim3 blk(128);
    a.vpart = e->vpart;
    a.nparts = (e->D + 3) / 4;
    a.ema_new = e->ema_new;
    a.ffn_inv = e->ffn_inv;
    const size_t attn_sm = (size_t)2 * kB1Chunk * (e->HD + 4) * 4;
    // FFN1 grid: enough warps to cover the hidden units of ~4 experts once
    int n_sm = 148;
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, e->ctx->device);
    const int ffn1_grid = 2 * n_sm;
    for (int l = 0; l < e->L; l++) {
        LayerDev &ly = e->layers[l];
        a.l = l;
        a.attn_norm = ly.attn_norm; a.ffn_norm = ly.ffn_norm; a.wqkv = ly.wqkv; a.wo = ly.wo; a.w_vote = ly.w_vote;
        a.alive = e->alive_dev + (size_t)l * kMaxE; a.temperature = ly.temperature;
        a.gu_tab = e->gu_tab + (size_t)l * kMaxE; a.dn_tab = e->dn_tab + (size_t)l * kMaxE;
        a.kc = e->kc + (size_t)l * e->max_seq * e->kd; a.vc = e->vc + (size_t)l * e->max_seq * e->kd;
        a.tr_k = e->tr_k; a.tr_sel = e->tr_sel; a.tr_w = e->tr_w; a.tr_ema = e->tr_ema;
        a.embed = l == 0;
        a.combine = 0;
        a.x = e->x;
        NV_SWITCH(nv, k_b1_qkv, dim3((e->qkvd + 3) / 4), blk, a);
        dim3 ga((e->max_seq + kB1Chunk - 1) / kB1Chunk, e->KVH);
        if (e->HD == 64) launch_pdl_sm(e, k_b1_attn<64>, ga, blk, attn_sm, a);
        else launch_pdl_sm(e, k_b1_attn<128>, ga, blk, attn_sm, a);
        if (e->HD == 64) {
            WO_SWITCH(nv, 64, dim3((e->D + 3) / 4), blk, a);
        } else {
            WO_SWITCH(nv, 128, dim3((e->D + 3) / 4), blk, a);
        }
        NV_SWITCH(nv, k_b1_ffn1, dim3(ffn1_grid), blk, a);
        NH_SWITCH(nh, k_b1_ffn2, dim3((e->D + 3) / 4, std::max(1, e->n_alive[l])), blk, a);
    }
    a.l = e->L;
    a.combine = 0;
    a.embed = 0;
    a.x = e->x;
    NV_SWITCH(nv, k_b1_lmhead, dim3(2 * n_sm), blk, a);
    if (!a.greedy_pick) jdg_launch_pick(e, 1);
}


// ------------------------------------------------------------------------------------
// Batch-1 persistent step (jdg_b1p.cuh): one cooperative launch per decode step.
template <int NV, int NH>
static cudaError_t b1p_prepare(size_t smem, int *blocks_per_sm) {
    cudaError_t r = cudaFuncSetAttribute(k_b1_step<NV, NH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (r != cudaSuccess) return r;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, k_b1_step<NV, NH>, kPThreads, smem);
}
template <int NV, int NH>
static void b1p_launch(jdg_engine *e, const B1PArgs &a, size_t smem) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(e->b1p_grid);
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = e->st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, k_b1_step<NV, NH>, a);
    e->launches++;
}

static int b1p_variant(const jdg_engine *e) {
    const int nv = e->D / 128, nh = e->hidden / 128;
    if (nv == 2 && nh == 3) return 0;
    if (nv == 4 && nh == 6) return 1;
    if (nv == 6 && nh == 9) return 2;
    return -1;
}

static size_t b1p_smem_bytes(const jdg_engine *e, int grid) {
    const int rq = (e->qkvd + grid - 1) / grid, rd = (e->D + grid - 1) / grid;
    return (size_t)b1p_smem(e->D, e->Hh, e->hidden, e->kmax, e->max_seq / kPChunk + 1, rq, rd).total * 4;
}

// Whether the persistent step serves this engine (decided once): shapes it is written for,
// every CTA resident on its own SM (cooperative launch), one attention item per CTA.
static bool b1p_usable(jdg_engine *e) {
    if (e->b1p_grid > 0) return true;
    if (e->b1p_grid < 0 || e->force_chain || !e->b1p_layers) return false;
    e->b1p_grid = -1;
    const int var = b1p_variant(e);
    if (var < 0 || e->HD != kPHD || e->qd != e->D || e->max_seq > 1024 || e->Hh % e->KVH ||
        e->Hh / e->KVH > kPMaxHG || e->L > JD_MAX_LAYERS)
        return false;
    int dev = e->ctx->device, n_sm = 0, coop = 0;
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
    if (!coop || n_sm < 1 || e->KVH * (e->max_seq / kPChunk + 1) > n_sm) return false;
    const size_t smem = b1p_smem_bytes(e, n_sm);
    int per_sm = 0;
    cudaError_t r = var == 0 ? b1p_prepare<2, 3>(smem, &per_sm)
                  : var == 1 ? b1p_prepare<4, 6>(smem, &per_sm)
                             : b1p_prepare<6, 9>(smem, &per_sm);
    if (r != cudaSuccess || per_sm < 1) {
        cudaGetLastError();
        return false;
    }
    e->b1p_grid = n_sm;
    return true;
}

static void enqueue_own_step_b1p(jdg_engine *e) {
    B1PArgs a = {};
    const int G = e->b1p_grid;
    a.layers = (const char *)e->b1p_layers;
    a.tok_emb = e->tok_emb; a.output = e->output; a.output_norm = e->output_norm;
    a.rope_cos = e->rope_cos; a.rope_sin = e->rope_sin;
    a.V = e->V; a.D = e->D; a.H = e->Hh; a.KVH = e->KVH; a.hidden = e->hidden; a.qkvd = e->qkvd;
    a.max_seq = e->max_seq; a.L = e->L; a.kmax = e->kmax; a.nch_max = e->max_seq / kPChunk + 1;
    a.eps = e->eps; a.scale = 1.0f / sqrtf((float)e->HD); a.clamp = e->clamp;
    a.inv_clamp = e->clamp > 0 ? 1.0f / e->clamp : 0.f;
    a.tok = e->tok; a.pos = e->pos; a.x = e->x; a.qkv = e->qkv; a.part = e->part; a.vpart = e->vpart;
    a.hbuf = e->hbuf; a.logits = e->logits; a.kc = e->kc; a.vc = e->vc; a.consensus = e->consensus;
    a.tr_k = e->tr_k; a.tr_sel = e->tr_sel; a.tr_w = e->tr_w; a.tr_ema = e->tr_ema;
    a.bar = e->tickets + 1000; a.ticket = e->tickets + 1001;
    a.amax_v = e->amax_v; a.amax_i = e->amax_i; a.stats = e->stats;
    a.tok_out = e->tok; a.plen = e->plen; a.prompt = e->prompt; a.hist = e->hist; a.hist_n = e->hist_n;
    a.next_out = e->next_out; a.Hmax = e->Hmax; a.greedy_pick = e->temp <= 0.f; a.err = e->err;
    a.tl = e->timeline;
    a.rq = (e->qkvd + G - 1) / G;
    a.rd = (e->D + G - 1) / G;
    const size_t smem = b1p_smem_bytes(e, G);
    cudaMemsetAsync(a.bar, 0, 4, e->st);
    switch (b1p_variant(e)) {
    case 0: b1p_launch<2, 3>(e, a, smem); break;
    case 1: b1p_launch<4, 6>(e, a, smem); break;
    default: b1p_launch<6, 9>(e, a, smem); break;
    }
    if (!a.greedy_pick) jdg_launch_pick(e, 1);
}

static void own_batch_layers(jdg_engine *e, int B, int prefill_slot);

// One own-model decode step for slots 0..B-1 (forward_token, janusdoe.c:879-934, then
// the next-token pick).
static void enqueue_own_step(jdg_engine *e, int B) {
    if (B == 1 && !e->force_generic && b1p_usable(e)) {
        enqueue_own_step_b1p(e);
        return;
    }
    if (B == 1 && b1_shape_ok(e) && !e->force_generic) {
        enqueue_own_step_b1(e);
        return;
    }
    own_batch_layers(e, B, -1);
    const int D = e->D, V = e->V;
    if (B == 1) {
        launch_gemv1(e, EPI_STORE, e->output, V, D, e->x, e->output_norm, 1, e->logits);
    } else {
        if (e->tc_ok) {  // final norm straight into the LM head's activation blocks
            k_tc_norm_prep<<<B, 256, 0, e->st>>>(e->x, e->output_norm, D, e->eps, e->tc_xt);
            e->launches++;
            launch_tc(e, e->tc_out_tab, 1, e->xb, 0, D, nullptr, 0, nullptr, B, B, V, D, e->logits, V, 0, EPI_STORE, 1.f,
                      0, 1);
        } else {
            k_rmsnorm<<<B, 256, 0, e->st>>>(e->x, e->output_norm, e->xb, D, e->eps);
            e->launches++;
            SgemmArgs a = {};
            a.A = e->xb; a.lda = D; a.M = B; a.W = e->output; a.N = V; a.K = D; a.C = e->logits; a.ldc = V;
            launch_sgemm<EPI_STORE>(e, a, B, 1);
        }
    }
    jdg_launch_pick(e, B);
}

// Embedding and every layer for B rows (sequences at one position each, or, with
// prefill_slot >= 0, the prompt tokens of that sequence at positions 0..B-1, whose elections
// take the EMA as a scan over the tokens in order).
static void own_batch_layers(jdg_engine *e, int B, int prefill_slot) {
    const int D = e->D, H = e->hidden, L = e->L, V = e->V, qd = e->qd;
    const float scale = 1.0f / sqrtf((float)e->HD);
    k_embed<<<B, 256, 0, e->st>>>(e->tok_emb, V, D, e->tok, e->x, e->err);
    e->launches++;
    for (int l = 0; l < L; l++) {
        LayerDev &ly = e->layers[l];
        // split-K partials of q/k/v and Wo summed by their consumers (rope, election)
        SplitPart qsp{nullptr, 1, 1}, wsp{nullptr, 1, 1};
        if (B == 1) {
            launch_gemv1(e, EPI_STORE, ly.wqkv, e->qkvd, D, e->x, ly.attn_norm, 1, e->qkv);
        } else {
            if (e->tc_ok) {  // attention norm straight into the q/k/v product's activation blocks
                k_tc_norm_prep<<<B, 256, 0, e->st>>>(e->x, ly.attn_norm, D, e->eps, e->tc_xt);
                e->launches++;
                launch_tc(e, ly.tc_wqkv_tab, 1, e->xb, 0, D, nullptr, 0, nullptr, B, B, e->qkvd, D, e->qkv, e->qkvd, 0,
                          EPI_STORE, 1.f, 0, 1, &qsp);
            } else {
                k_rmsnorm<<<B, 256, 0, e->st>>>(e->x, ly.attn_norm, e->xb, D, e->eps);
                e->launches++;
                SgemmArgs a = {};
                a.A = e->xb; a.lda = D; a.M = B; a.W = ly.wqkv; a.N = e->qkvd; a.K = D; a.C = e->qkv; a.ldc = e->qkvd;
                launch_sgemm<EPI_STORE>(e, a, B, 1);
            }
        }
        jdg_launch_rope(e, l, B, qsp);
        launch_attention(e, l, B, scale, 1.0f, B > 1 && e->tc_ok);
        if (B == 1) {
            launch_gemv1(e, EPI_ADD, ly.wo, D, qd, e->att, nullptr, 0, e->x);
        } else if (e->tc_ok) {  // the attention merge wrote the activation blocks
            launch_tc(e, ly.tc_wo_tab, 1, e->att, 0, qd, nullptr, 0, nullptr, B, B, D, qd, e->x, D, 0, EPI_ADD, 1.f, 0,
                      1, &wsp);
        } else {
            SgemmArgs a = {};
            a.A = e->att; a.lda = qd; a.M = B; a.W = ly.wo; a.N = D; a.K = qd; a.C = e->x; a.ldc = D;
            launch_sgemm<EPI_ADD>(e, a, B, 1);
        }
        if (prefill_slot < 0) {
            jdg_launch_elect(e, l, B, e->x, ly.ffn_norm, ly.w_vote, e->alive_dev + (size_t)l * kMaxE, ly.temperature, 0,
                             wsp);
        } else {
            ElectArgs a = {};
            a.x = e->x; a.norm_w = ly.ffn_norm; a.eps = e->eps; a.D = D; a.host = 0; a.w_vote = ly.w_vote;
            a.alive = e->alive_dev + (size_t)l * kMaxE; a.temperature = ly.temperature; a.consensus = e->consensus;
            a.L = L; a.l = l; a.xb = e->xb; a.kcnt = e->kcnt; a.sel = e->sel; a.selw = e->selw; a.tr_k = e->tr_k;
            a.tr_sel = e->tr_sel; a.tr_w = e->tr_w; a.tr_ema = e->tr_ema;
            a.prefill = 1; a.pf_votes = e->pf_votes; a.pf_cs = e->pf_cs;
            a.pf_cons = e->consensus + (size_t)prefill_slot * L + l;
            a.sp = wsp;
            a.x_out = e->x;
            k_elect<<<B, 256, (size_t)D * 4, e->st>>>(a);
            k_elect_scan<<<1, 256, (size_t)B * 4, e->st>>>(a, B);
            e->launches += 2;
        }
        const float *const *gu = e->gu_tab + (size_t)l * kMaxE;
        const float *const *dn = e->dn_tab + (size_t)l * kMaxE;
        if (e->n_alive[l] < 2) continue;  // parliament_elect returns 0 below MIN_EXPERTS
        if (B == 1) {
            k_route<<<1, 512, 0, e->st>>>(e->kcnt, e->sel, B, e->rcnt, e->ridx, e->pairrow, e->stats);
            e->launches++;
            dim3 g1((H + 3) / 4, e->n_alive[l]);
            k_expert_gu_b1<<<g1, 128, (size_t)D * 4, e->st>>>(gu, e->kcnt, e->sel, H, D, e->xb, e->hbuf, e->err);
            k_expert_down_b1<<<(D + 3) / 4, 128, (size_t)e->n_alive[l] * H * 4, e->st>>>(dn, e->kcnt, e->sel, e->selw, D,
                                                                                         H, e->hbuf, e->x);
            e->launches += 2;
        } else {
            k_route<<<1, 512, 0, e->st>>>(e->kcnt, e->sel, B, e->rcnt, e->ridx, e->pairrow, e->stats);
            if (e->tc_ok) {
                // segments = expert slots: gate/up of the routed rows of xb (gathered) stored as
                // interleaved (gate, up) rows [slot][B][2H]; down's activation prep applies
                // silu(gate) * up while it splits the operand
                launch_tc(e, ly.tc_gu, kMaxE, e->xb, 0, D, e->ridx, B, e->rcnt, 0, B, 2 * H, D, e->hbuf, 2 * H,
                          (long)B * 2 * H, EPI_STORE, 1.f);
                launch_tc(e, ly.tc_dn, kMaxE, e->hbuf, (long)B * 2 * H, 2 * H, nullptr, 0, e->rcnt, 0, B, D, H, e->ybuf,
                          D, (long)B * D, EPI_STORE, 1.f, 1);
            } else {
                SgemmArgs a = {};
                a.A = e->xb; a.lda = D; a.idx = e->ridx; a.ldi = B; a.cnt = e->rcnt; a.Wtab = gu; a.N = 2 * H; a.K = D;
                a.C = e->hbuf; a.ldc = H; a.c_seg_rows = B;
                launch_sgemm<EPI_SWIGLU>(e, a, B, kMaxE);
                SgemmArgs d = {};
                d.A = e->hbuf; d.lda = H; d.a_seg_rows = B; d.cnt = e->rcnt; d.Wtab = dn; d.N = D; d.K = H;
                d.C = e->ybuf; d.ldc = D; d.c_seg_rows = B;
                launch_sgemm<EPI_STORE>(e, d, B, kMaxE);
            }
            k_combine<<<B, 256, 0, e->st>>>(e->kcnt, e->selw, e->pairrow, e->ybuf, D, e->x);
            e->launches += 2;
        }
    }
}

static int enqueue_step(jdg_engine *e, int B) {
    if (e->kind == 0) enqueue_own_step(e, B);
    else return jdg_enqueue_host_step(e, B);
    return JD_OK;
}

// Capture one step for batch B into a CUDA graph (built once per B and sampling setting).
static int get_graph(jdg_engine *e, int B, cudaGraphExec_t *out) {
    auto it = e->graphs.find(B);
    if (it != e->graphs.end()) {
        *out = it->second;
        return JD_OK;
    }
    static bool attr_done = false;
    if (!attr_done) {
        CK(cudaFuncSetAttribute(k_gemv_f32<1, 1, EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        CK(cudaFuncSetAttribute(k_gemv_f32<1, 1, EPI_ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        CK(cudaFuncSetAttribute(k_expert_down_b1, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        CK(cudaFuncSetAttribute(k_expert_gu_b1, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        CK(cudaFuncSetAttribute(k_elect, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        CK(cudaFuncSetAttribute(k_b1_attn<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        CK(cudaFuncSetAttribute(k_b1_attn<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        int rc = jdg_host_set_attrs(e);
        if (rc != JD_OK) return rc;
        attr_done = true;
    }
    cudaGraph_t g;
    CK(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal));
    long long before = e->launches;
    int rc = enqueue_step(e, B);
    cudaError_t r = cudaStreamEndCapture(e->st, &g);
    if (rc != JD_OK) return rc;
    if (r != cudaSuccess) {
        jdg_set_err(e->ctx, "graph capture failed: %s", cudaGetErrorString(r));
        return JD_ECUDA;
    }
    cudaGraphExec_t ge;
    r = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (r != cudaSuccess) {
        jdg_set_err(e->ctx, "graph instantiate failed: %s", cudaGetErrorString(r));
        return JD_ECUDA;
    }
    e->launches_per_step[B] = e->launches - before;
    e->launches = before;
    e->graphs[B] = ge;
    *out = ge;
    return JD_OK;
}

static void drop_graphs(jdg_engine *e) {
    for (auto &kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
}
int jdg_host_drop_graphs(jdg_engine *e) {
    drop_graphs(e);
    return JD_OK;
}

static int check_err(jdg_engine *e) {
    int h = 0;
    if (e->pin_err) {  // a pinned destination keeps the copy asynchronous (no staging)
        CK(cudaMemcpyAsync(e->pin_err, e->err, 4, cudaMemcpyDeviceToHost, e->st));
        CK(cudaStreamSynchronize(e->st));
        h = *e->pin_err;
    } else {
        CK(cudaMemcpyAsync(&h, e->err, 4, cudaMemcpyDeviceToHost, e->st));
        CK(cudaStreamSynchronize(e->st));
    }
    if (h) {
        CK(cudaMemsetAsync(e->err, 0, 4, e->st));
        jdg_set_err(e->ctx, "device-side check failed (flags 0x%x: %s%s%s%s%s)", h, (h & JDG_ERR_TOKEN) ? "token " : "",
                    (h & JDG_ERR_POS) ? "position " : "", (h & JDG_ERR_ROUTE) ? "route " : "",
                    (h & JDG_ERR_SHAPE) ? "shape " : "", (h & JDG_ERR_TIMEOUT) ? "copy wait timed out" : "");
        return JD_ESTATE;
    }
    return JD_OK;
}

// ------------------------------------------------------------------------------------
extern "C" void jdg_engine_free(jdg_engine *e) {
    if (!e) return;
    cudaSetDevice(e->ctx->device);
    if (e->st) cudaStreamSynchronize(e->st);
    drop_graphs(e);
    jdg_host_release(e);
    for (void *p : e->allocs) cudaFree(p);
    if (e->pin_tok) cudaFreeHost(e->pin_tok);
    if (e->ev0) cudaEventDestroy(e->ev0);
    if (e->ev1) cudaEventDestroy(e->ev1);
    if (e->st) cudaStreamDestroy(e->st);
    delete e;
}

extern "C" int jdg_set_sampling(jdg_engine *e, float temperature, int top_k) {
    if (!e || top_k < 0) return JD_EINVAL;
    if (temperature != e->temp || top_k != e->top_k) drop_graphs(e);
    e->temp = temperature;
    e->top_k = top_k;
    return JD_OK;
}

extern "C" int jdg_reset(jdg_engine *e, int slot) {
    if (!e || slot >= e->B_max || slot < -1) return JD_EINVAL;
    cudaSetDevice(e->ctx->device);
    int s0 = slot < 0 ? 0 : slot, s1 = slot < 0 ? e->B_max : slot + 1, n = s1 - s0;
    CK(cudaMemsetAsync(e->kc + (size_t)s0 * e->kv_bstride, 0, (size_t)n * e->kv_bstride * 4, e->st));
    CK(cudaMemsetAsync(e->vc + (size_t)s0 * e->kv_bstride, 0, (size_t)n * e->kv_bstride * 4, e->st));
    std::vector<float> cons((size_t)n * e->L);
    for (int b = 0; b < n; b++)
        for (int l = 0; l < e->L; l++) cons[(size_t)b * e->L + l] = e->layer_consensus[l];
    CK(cudaMemcpyAsync(e->consensus + (size_t)s0 * e->L, cons.data(), cons.size() * 4, cudaMemcpyHostToDevice, e->st));
    CK(cudaMemsetAsync(e->plen + s0, 0, n * 4, e->st));
    CK(cudaMemsetAsync(e->hist_n + s0, 0, n * 4, e->st));
    CK(cudaMemsetAsync(e->pos + s0, 0, n * 4, e->st));
    CK(cudaStreamSynchronize(e->st));
    return JD_OK;
}

extern "C" int jdg_set_prompt(jdg_engine *e, int B, const int *tokens, int P, const int *len, const uint64_t *rng) {
    if (!e || B < 1 || B > e->B_max || !tokens || !len || P < 1 || P > e->Pmax) return JD_EINVAL;
    cudaSetDevice(e->ctx->device);
    for (int b = 0; b < B; b++)
        if (len[b] < 1 || len[b] > P) {
            jdg_set_err(e->ctx, "prompt length %d of slot %d outside [1, %d]", len[b], b, P);
            return JD_EINVAL;
        }
    std::vector<int> pr((size_t)B * e->Pmax, 0), t0(B), p0(B, 0);
    for (int b = 0; b < B; b++) {
        memcpy(&pr[(size_t)b * e->Pmax], tokens + (size_t)b * P, (size_t)len[b] * 4);
        t0[b] = tokens[(size_t)b * P];
    }
    e->prompt_host = pr;
    e->plen_host.assign(len, len + B);
    CK(cudaMemcpyAsync(e->prompt, pr.data(), pr.size() * 4, cudaMemcpyHostToDevice, e->st));
    CK(cudaMemcpyAsync(e->plen, len, B * 4, cudaMemcpyHostToDevice, e->st));
    CK(cudaMemcpyAsync(e->tok, t0.data(), B * 4, cudaMemcpyHostToDevice, e->st));
    CK(cudaMemcpyAsync(e->pos, p0.data(), B * 4, cudaMemcpyHostToDevice, e->st));
    if (rng) CK(cudaMemcpyAsync(e->rng, rng, B * 8, cudaMemcpyHostToDevice, e->st));
    CK(cudaMemsetAsync(e->hist_n, 0, B * 4, e->st));
    CK(cudaStreamSynchronize(e->st));
    return JD_OK;
}

extern "C" int jdg_run(jdg_engine *e, int B, int n_steps) {
    if (!e || B < 1 || B > e->B_max || n_steps < 0) return JD_EINVAL;
    cudaSetDevice(e->ctx->device);
    cudaGraphExec_t ge;
    int rc = get_graph(e, B, &ge);
    if (rc != JD_OK) return rc;
    CK(cudaEventRecord(e->ev0, e->st));
    for (int i = 0; i < n_steps; i++) CK(cudaGraphLaunch(ge, e->st));
    CK(cudaEventRecord(e->ev1, e->st));
    CK(cudaEventSynchronize(e->ev1));
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, e->ev0, e->ev1));
    e->last_ms = ms;
    e->launches += (long long)n_steps * e->launches_per_step[B];
    return check_err(e);
}

// ------------------------------------------------------------------------------------
// Prompt prefill of the own model: the prompt tokens of a sequence go through the layers as
// one batch of rows (GEMMs over all tokens, causal attention over the slot's KV cache), and
// each layer's elections take the EMA as an ordered scan over the tokens, so that k, the
// elected experts and the EMA are those of token-by-token decoding (janusdoe.c:3660).
static int pf_alloc(jdg_engine *e) {
    if (e->pf_x) return JD_OK;
    const size_t P = e->max_seq, D = e->D, H = e->hidden, L = e->L;
    DALLOC(e->pf_x, P * D * 4);
    DALLOC(e->pf_xb, P * D * 4);
    DALLOC(e->pf_qkv, P * e->qkvd * 4);
    DALLOC(e->pf_att, P * e->qd * 4);
    DALLOC(e->pf_part, P * e->Hh * e->nchunk * (e->HD + 2) * 4);
    DALLOC(e->pf_hbuf, (size_t)kMaxE * P * 2 * H * 4);
    DALLOC(e->pf_ybuf, (size_t)kMaxE * P * D * 4);
    DALLOC(e->pf_kcnt, P * 4);
    DALLOC(e->pf_sel, P * kMaxE * 4);
    DALLOC(e->pf_selw, P * kMaxE * 4);
    DALLOC(e->pf_rcnt, kMaxE * 4);
    DALLOC(e->pf_ridx, kMaxE * P * 4);
    DALLOC(e->pf_pairrow, P * kMaxE * 4);
    DALLOC(e->pf_pos, P * 4);
    DALLOC(e->pf_votes, P * kMaxE * 4);
    DALLOC(e->pf_cs, P * 4);
    DALLOC(e->pf_tr_k, P * L * 4);
    DALLOC(e->pf_tr_sel, P * L * kMaxE * 4);
    DALLOC(e->pf_tr_w, P * L * kMaxE * 4);
    DALLOC(e->pf_tr_ema, P * L * 4);
    std::vector<int> iota(P);
    for (size_t i = 0; i < P; i++) iota[i] = (int)i;
    CK(cudaMemcpy(e->pf_pos, iota.data(), P * 4, cudaMemcpyHostToDevice));
    CK(cudaMemset(e->pf_hbuf, 0, (size_t)kMaxE * P * 2 * H * 4));
    CK(cudaMemset(e->pf_ybuf, 0, (size_t)kMaxE * P * D * 4));
    return JD_OK;
}

// The batch rows of the engine, swapped for the prefill's while it runs.
struct OwnRows {
    int *tok, *pos, *kcnt, *sel, *rcnt, *ridx, *pairrow, *tr_k, *tr_sel;
    float *x, *xb, *qkv, *att, *part, *hbuf, *ybuf, *selw, *kc, *vc, *tr_w, *tr_ema;
    long kv_bstride;
};
static OwnRows rows_of(const jdg_engine *e) {
    return OwnRows{e->tok, e->pos, e->kcnt, e->sel, e->rcnt, e->ridx, e->pairrow, e->tr_k, e->tr_sel,
                   e->x, e->xb, e->qkv, e->att, e->part, e->hbuf, e->ybuf, e->selw, e->kc, e->vc, e->tr_w,
                   e->tr_ema, e->kv_bstride};
}
static void set_rows(jdg_engine *e, const OwnRows &r) {
    e->tok = r.tok; e->pos = r.pos; e->kcnt = r.kcnt; e->sel = r.sel; e->rcnt = r.rcnt; e->ridx = r.ridx;
    e->pairrow = r.pairrow; e->tr_k = r.tr_k; e->tr_sel = r.tr_sel; e->x = r.x; e->xb = r.xb; e->qkv = r.qkv;
    e->att = r.att; e->part = r.part; e->hbuf = r.hbuf; e->ybuf = r.ybuf; e->selw = r.selw; e->kc = r.kc;
    e->vc = r.vc; e->tr_w = r.tr_w; e->tr_ema = r.tr_ema; e->kv_bstride = r.kv_bstride;
}

extern "C" int jdg_prefill(jdg_engine *e, int B) {
    if (!e || B < 1 || B > e->B_max || (int)e->plen_host.size() < B) return JD_EINVAL;
    if (e->kind != 0) {
        jdg_set_err(e->ctx, "jdg_prefill: the host model's prompts run through jdg_run");
        return JD_EUNSUPPORTED;
    }
    cudaSetDevice(e->ctx->device);
    int rc = pf_alloc(e);
    if (rc != JD_OK) return rc;
    CK(cudaEventRecord(e->ev0, e->st));
    const OwnRows saved = rows_of(e);
    for (int b = 0; b < B; b++) {
        const int n = e->plen_host[b] - 1;  // every prompt token but the last
        if (n >= 1) {
            OwnRows r = saved;
            r.tok = e->prompt + (size_t)b * e->Pmax;
            r.pos = e->pf_pos;
            r.kcnt = e->pf_kcnt; r.sel = e->pf_sel; r.selw = e->pf_selw; r.rcnt = e->pf_rcnt; r.ridx = e->pf_ridx;
            r.pairrow = e->pf_pairrow; r.tr_k = e->pf_tr_k; r.tr_sel = e->pf_tr_sel; r.tr_w = e->pf_tr_w;
            r.tr_ema = e->pf_tr_ema; r.x = e->pf_x; r.xb = e->pf_xb; r.qkv = e->pf_qkv; r.att = e->pf_att;
            r.part = e->pf_part; r.hbuf = e->pf_hbuf; r.ybuf = e->pf_ybuf;
            r.kc = saved.kc + (size_t)b * saved.kv_bstride;
            r.vc = saved.vc + (size_t)b * saved.kv_bstride;
            r.kv_bstride = 0;  // every row is a position of this one sequence
            set_rows(e, r);
            own_batch_layers(e, n, b);
            set_rows(e, saved);
            e->pf_last_n = n;
        }
        // the slot continues at the last prompt token, as after n decode steps
        const int last = e->prompt_host[(size_t)b * e->Pmax + n];
        CK(cudaMemcpyAsync(e->tok + b, &last, 4, cudaMemcpyHostToDevice, e->st));
        CK(cudaMemcpyAsync(e->pos + b, &n, 4, cudaMemcpyHostToDevice, e->st));
        CK(cudaStreamSynchronize(e->st));  // `last` and `n` are stack values
    }
    CK(cudaEventRecord(e->ev1, e->st));
    CK(cudaEventSynchronize(e->ev1));
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, e->ev0, e->ev1));
    e->last_ms = ms;
    return check_err(e);
}

extern "C" int jdg_get_prefill_trace(jdg_engine *e, int n, jdg_trace *tr) {
    if (!e || !tr || n < 1 || n > e->pf_last_n || !e->pf_tr_k) return JD_EINVAL;
    cudaSetDevice(e->ctx->device);
    const size_t L = e->L;
    if (tr->k) CK(cudaMemcpy(tr->k, e->pf_tr_k, (size_t)n * L * 4, cudaMemcpyDeviceToHost));
    if (tr->sel) CK(cudaMemcpy(tr->sel, e->pf_tr_sel, (size_t)n * L * kMaxE * 4, cudaMemcpyDeviceToHost));
    if (tr->w) CK(cudaMemcpy(tr->w, e->pf_tr_w, (size_t)n * L * kMaxE * 4, cudaMemcpyDeviceToHost));
    if (tr->ema) CK(cudaMemcpy(tr->ema, e->pf_tr_ema, (size_t)n * L * 4, cudaMemcpyDeviceToHost));
    return JD_OK;
}

extern "C" int jdg_last_run_ms(jdg_engine *e, float *ms) {
    if (!e || !ms) return JD_EINVAL;
    *ms = e->last_ms;
    return JD_OK;
}

extern "C" int jdg_get_stats(jdg_engine *e, uint64_t *out3) {
    if (!e || !out3) return JD_EINVAL;
    cudaSetDevice(e->ctx->device);
    unsigned long long h[3];
    CK(cudaMemcpyAsync(h, e->stats, 3 * 8, cudaMemcpyDeviceToHost, e->st));
    CK(cudaStreamSynchronize(e->st));
    for (int i = 0; i < 3; i++) out3[i] = h[i];
    return JD_OK;
}

extern "C" int jdg_reset_stats(jdg_engine *e) {
    if (!e) return JD_EINVAL;
    cudaSetDevice(e->ctx->device);
    CK(cudaMemsetAsync(e->stats, 0, 4 * 8, e->st));
    CK(cudaStreamSynchronize(e->st));
    return JD_OK;
}

// Debug: enable (n_slots > 0) or read the batch-1 kernel timeline.  Kernel chain:
// out[slot*3 + {0,1,2}] = earliest CTA entry, earliest return from the dependency wait,
// latest CTA exit (ns).  Persistent step: slot 1 + 5*layer + phase holds {earliest phase
// start, -, latest phase end} and slot 256 + the same index {-, -, latest phase start}.
extern "C" int jdg_debug_timeline(jdg_engine *e, int n_slots, uint64_t *out) {
    if (!e || n_slots < 0 || n_slots > 512) return JD_EINVAL;
    cudaSetDevice(e->ctx->device);
    if (!e->timeline) {
        DALLOC(e->timeline, (size_t)3 * 512 * 8);
        drop_graphs(e);
    }
    if (out) {
        CK(cudaMemcpyAsync(out, e->timeline, (size_t)3 * n_slots * 8, cudaMemcpyDeviceToHost, e->st));
        CK(cudaStreamSynchronize(e->st));
    }
    std::vector<unsigned long long> init(3 * 512);
    for (int i = 0; i < 512; i++) {
        init[3 * i] = ~0ull;
        init[3 * i + 1] = ~0ull;
        init[3 * i + 2] = 0;
    }
    CK(cudaMemcpyAsync(e->timeline, init.data(), init.size() * 8, cudaMemcpyHostToDevice, e->st));
    CK(cudaStreamSynchronize(e->st));
    return JD_OK;
}

extern "C" int jdg_launch_count(jdg_engine *e, long long *n) {
    if (!e || !n) return JD_EINVAL;
    *n = e->launches;
    return JD_OK;
}

extern "C" int jdg_get_state(jdg_engine *e, int B, int *tok, int *pos) {
    if (!e || B < 1 || B > e->B_max) return JD_EINVAL;
    cudaSetDevice(e->ctx->device);
    if (tok) CK(cudaMemcpyAsync(tok, e->tok, B * 4, cudaMemcpyDeviceToHost, e->st));
    if (pos) CK(cudaMemcpyAsync(pos, e->pos, B * 4, cudaMemcpyDeviceToHost, e->st));
    CK(cudaStreamSynchronize(e->st));
    return JD_OK;
}

extern "C" int jdg_get_history(jdg_engine *e, int B, int n, int *tokens) {
    if (!e || B < 1 || B > e->B_max || n < 0 || n > e->Hmax || !tokens) return JD_EINVAL;
    cudaSetDevice(e->ctx->device);
    std::vector<int> h((size_t)B * e->Hmax), hn(B);
    CK(cudaMemcpyAsync(h.data(), e->hist, h.size() * 4, cudaMemcpyDeviceToHost, e->st));
    CK(cudaMemcpyAsync(hn.data(), e->hist_n, B * 4, cudaMemcpyDeviceToHost, e->st));
    CK(cudaStreamSynchronize(e->st));
    for (int b = 0; b < B; b++) {
        int cnt = hn[b] < e->Hmax ? hn[b] : e->Hmax;
        for (int i = 0; i < n; i++) {
            int src = cnt - n + i;
            tokens[(size_t)b * n + i] = src >= 0 ? h[(size_t)b * e->Hmax + src] : -1;
        }
    }
    return JD_OK;
}

extern "C" int jdg_get_logits(jdg_engine *e, int B, float *logits) {
    if (!e || B < 1 || B > e->B_max || !logits) return JD_EINVAL;
    cudaSetDevice(e->ctx->device);
    CK(cudaMemcpyAsync(logits, e->logits, (size_t)B * e->ldl * 4, cudaMemcpyDeviceToHost, e->st));
    CK(cudaStreamSynchronize(e->st));
    return JD_OK;
}

extern "C" int jdg_get_trace(jdg_engine *e, int B, jdg_trace *t) {
    if (!e || B < 1 || B > e->B_max || !t) return JD_EINVAL;
    cudaSetDevice(e->ctx->device);
    const size_t n = (size_t)B * e->L;
    if (t->k) CK(cudaMemcpyAsync(t->k, e->tr_k, n * 4, cudaMemcpyDeviceToHost, e->st));
    if (t->ema) CK(cudaMemcpyAsync(t->ema, e->tr_ema, n * 4, cudaMemcpyDeviceToHost, e->st));
    if (t->sel) CK(cudaMemcpyAsync(t->sel, e->tr_sel, n * kMaxE * 4, cudaMemcpyDeviceToHost, e->st));
    if (t->w) CK(cudaMemcpyAsync(t->w, e->tr_w, n * kMaxE * 4, cudaMemcpyDeviceToHost, e->st));
    CK(cudaStreamSynchronize(e->st));
    return JD_OK;
}

extern "C" int jdg_step(jdg_engine *e, int B, const int *tok, const int *pos, uint64_t *rng, int *next_tok, float *logits,
                        jdg_trace *trace) {
    if (!e || B < 1 || B > e->B_max || !tok || !pos) return JD_EINVAL;
    for (int b = 0; b < B; b++) {
        if (pos[b] < 0 || pos[b] >= e->max_seq) {
            jdg_set_err(e->ctx, "position %d of slot %d outside [0, %d)", pos[b], b, e->max_seq);
            return JD_EINVAL;
        }
        if (tok[b] < 0 || (e->kind == 0 && tok[b] >= e->V)) {
            jdg_set_err(e->ctx, "token %d of slot %d outside [0, %d)", tok[b], b, e->V);
            return JD_EINVAL;
        }
    }
    cudaSetDevice(e->ctx->device);
    cudaGraphExec_t ge;
    int rc = get_graph(e, B, &ge);
    if (rc != JD_OK) return rc;
    memcpy(e->pin_tok, tok, B * 4);
    memcpy(e->pin_pos, pos, B * 4);
    CK(cudaMemcpyAsync(e->tok, e->pin_tok, B * 4, cudaMemcpyHostToDevice, e->st));
    CK(cudaMemcpyAsync(e->pos, e->pin_pos, B * 4, cudaMemcpyHostToDevice, e->st));
    CK(cudaMemsetAsync(e->plen, 0, B * 4, e->st));
    if (rng) CK(cudaMemcpyAsync(e->rng, rng, B * 8, cudaMemcpyHostToDevice, e->st));
    CK(cudaEventRecord(e->ev0, e->st));
    CK(cudaGraphLaunch(ge, e->st));
    CK(cudaEventRecord(e->ev1, e->st));
    e->launches += e->launches_per_step[B];
    CK(cudaMemcpyAsync(e->pin_next, e->next_out, B * 4, cudaMemcpyDeviceToHost, e->st));
    if (rng) CK(cudaMemcpyAsync(rng, e->rng, B * 8, cudaMemcpyDeviceToHost, e->st));
    if (logits) CK(cudaMemcpyAsync(logits, e->logits, (size_t)B * e->ldl * 4, cudaMemcpyDeviceToHost, e->st));
    rc = check_err(e);
    if (rc != JD_OK) return rc;
    if (next_tok) memcpy(next_tok, e->pin_next, B * 4);
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, e->ev0, e->ev1));
    e->last_ms = ms;
    if (trace) return jdg_get_trace(e, B, trace);
    return JD_OK;
}

extern "C" int jdg_profile_step(jdg_engine *e, int B, float *ms_by_kernel, int max_kernels, int *n_kernels,
                                const char **names) {
    (void)e; (void)B; (void)ms_by_kernel; (void)max_kernels; (void)names;
    if (n_kernels) *n_kernels = 0;
    return JD_EUNSUPPORTED;
}

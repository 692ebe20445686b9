/*
 * jd_oracle.c — CPU restatement of the janus.DoE decode path (TEST INFRASTRUCTURE ONLY).
 *
 * Restates, in the reference's operation order, the functions on the token loop
 * of janusdoe.c:
 *   own model : config_from_depth, rng, rmsnorm/matvec/softmax_n/apply_rope,
 *               parliament_elect, forward_token, sample
 *   host GGUF : jd_f16_to_f32, jd_dequant_*, jd_pq_*_rows, jd_qmatvec,
 *               gguf_host_load (decode-relevant parts), host_parliament_elect,
 *               gguf_host_forward
 * Build with plain `-O3` (no -march, no -ffast-math): the x86-64 baseline has no FMA,
 * so the compiler neither contracts nor reorders, and the results equal the reference
 * built the same way, bit for bit.
 *
 * Parity pin: tests/test_oracle_pin.py runs this file against the reference source
 * compiled by oracle/Makefile (oracle/_ref/libjdref.so) and tests/test_oracle_golden.py
 * against the fixtures in tests/golden/ that that build produced.
 *
 * Only tests, the smoke check and the benchmark's CPU-baseline leg load this code.
 */
#include "jd_oracle.h"
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#include <pthread.h>
#include <unistd.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>

/* ============================ RNG ======================================= */

/* Seed mapping used by every implementation of the synthetic workloads: the
 * reference's xorshift64 has 0 as a fixed point, so a user seed is first mixed
 * by splitmix64 (Steele, Lea & Flood 2014) and a zero result is replaced by 1. */
uint64_t jdo_splitmix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    z = z ^ (z >> 31);
    return z ? z : 1;
}
/* janusdoe.c:191 rng_next: xorshift64 with shifts 13, 7, 17 */
uint64_t jdo_rng_next(uint64_t *s) {
    uint64_t x = *s;
    x ^= x << 13; x ^= x >> 7; x ^= x << 17;
    *s = x; return x;
}
/* janusdoe.c:192 rand_uniform: low 31 bits over 0x7FFFFFFF, in float */
float jdo_rand_uniform(uint64_t *s) {
    return (float)(jdo_rng_next(s) & 0x7FFFFFFF) / (float)0x7FFFFFFF;
}
/* janusdoe.c:193 rand_normal: Box-Muller, cosine branch, u1 floored at 1e-10 */
float jdo_rand_normal(uint64_t *s) {
    float u1 = jdo_rand_uniform(s), u2 = jdo_rand_uniform(s);
    if (u1 < 1e-10f) u1 = 1e-10f;
    return sqrtf(-2.0f * logf(u1)) * cosf(6.2831853f * u2);
}

/* ============================ threads =================================== */
static int g_threads = 0;
void jdo_set_threads(int n) { g_threads = n; }
static int jdo_nthreads(void) {
    if (g_threads > 0) return g_threads > 64 ? 64 : g_threads;
    long c = sysconf(_SC_NPROCESSORS_ONLN);
    int n = c > 0 ? (int)c : 1;
    return n > 64 ? 64 : n;
}
typedef void (*jdo_rows_fn)(float *, const uint8_t *, const float *, int, int, int);
typedef struct { jdo_rows_fn fn; float *out; const uint8_t *W; const float *x; int r0, r1, c; } jdo_work;
static void *jdo_worker(void *a) { jdo_work *w = (jdo_work *)a; w->fn(w->out, w->W, w->x, w->r0, w->r1, w->c); return NULL; }
/* Rows are independent and each is summed sequentially, so splitting rows over
 * threads (as janusdoe.c:2685-2694 does) leaves every output bit unchanged. */
static void jdo_run_rows(jdo_rows_fn fn, float *out, const uint8_t *W, const float *x, int r, int c) {
    int nt = jdo_nthreads(); if (nt > r) nt = r;
    if (nt <= 1 || (long)r * c < (1L << 20)) { fn(out, W, x, 0, r, c); return; }
    pthread_t th[64]; jdo_work wk[64]; int chunk = (r + nt - 1) / nt, n = 0;
    for (int t = 0; t < nt; t++) {
        int r0 = t * chunk, r1 = r0 + chunk; if (r0 >= r) break; if (r1 > r) r1 = r;
        wk[t] = (jdo_work){fn, out, W, x, r0, r1, c};
        pthread_create(&th[t], NULL, jdo_worker, &wk[t]); n++;
    }
    for (int t = 0; t < n; t++) pthread_join(th[t], NULL);
}

/* ============================ f32 math ================================== */
/* janusdoe.c:504 rmsnorm: out = x * (1/sqrt(mean(x^2)+eps)) * w */
static void jdo_rmsnorm(float *out, const float *x, const float *w, int d, float eps) {
    float ss = 0; for (int i = 0; i < d; i++) ss += x[i] * x[i];
    float inv = 1.0f / sqrtf(ss / d + eps);
    for (int i = 0; i < d; i++) out[i] = x[i] * inv * w[i];
}
/* janusdoe.c:517 matvec (plain build): one sequential f32 accumulator per row */
static void jdo_f32_rows(float *out, const uint8_t *Wb, const float *x, int r0, int r1, int c) {
    const float *W = (const float *)Wb;
    for (int i = r0; i < r1; i++) { float s = 0; const float *row = W + (size_t)i * c; for (int j = 0; j < c; j++) s += row[j] * x[j]; out[i] = s; }
}
void jdo_matvec(float *out, const float *W, const float *x, int r, int c) {
    jdo_run_rows(jdo_f32_rows, out, (const uint8_t *)W, x, r, c);
}
/* janusdoe.c:534 softmax_n */
static void jdo_softmax(float *x, int n) {
    float mx = x[0]; for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    float s = 0; for (int i = 0; i < n; i++) { x[i] = expf(x[i] - mx); s += x[i]; }
    for (int i = 0; i < n; i++) x[i] /= s;
}
/* janusdoe.c:536 apply_rope: NeoX-half pairing (i, i+hd/2) from the cos/sin cache */
static void jdo_rope_cache(float *v, int pos, const float *cc, const float *sc, int hd) {
    int h = hd / 2, off = pos * h;
    for (int i = 0; i < h; i++) {
        float x0 = v[i], x1 = v[i + h];
        v[i] = x0 * cc[off + i] - x1 * sc[off + i];
        v[i + h] = x0 * sc[off + i] + x1 * cc[off + i];
    }
}
/* janusdoe.c:498 silu_f */
static float jdo_silu(float x) { return x / (1.0f + expf(-x)); }

/* ============================ own model ================================= */

/* janusdoe.c:151-185 config_from_depth (decode-relevant fields) */
int jdo_config_from_depth(int depth, jdo_config *c) {
    memset(c, 0, sizeof(*c));
    c->depth = depth;
    c->dim = depth * 64; c->dim = ((c->dim + 63) / 64) * 64;
    if (c->dim < 128) c->dim = 128;
    if (c->dim > 768) c->dim = 768;
    c->head_dim = 64;
    c->n_heads = c->dim / c->head_dim; if (c->n_heads < 1) c->n_heads = 1;
    if (c->dim <= 384) c->n_kv_heads = c->n_heads;
    else {
        c->n_kv_heads = c->n_heads / 2; if (c->n_kv_heads < 1) c->n_kv_heads = 1;
        while (c->n_heads % c->n_kv_heads != 0 && c->n_kv_heads > 1) c->n_kv_heads--;
    }
    c->initial_experts = (depth <= 4) ? 4 : (depth <= 8) ? 6 : 8;
    c->hidden_dim = (int)(c->dim * 1.5f); c->hidden_dim = ((c->hidden_dim + 63) / 64) * 64;
    c->seq_len = 256; c->norm_eps = 1e-5f; c->rope_theta = 10000.0f; c->attn_clamp = 30.0f;
    c->active_depth = depth;
    c->vocab_size = 256 + 2 + (depth <= 4 ? 2000 : depth <= 8 ? 4000 : 8000);
    return 0;
}

/* Shapes follow janusdoe.c:744-776 init_weights: norms = 1, experts 0..initial-1 alive,
 * Parliament.consensus = 0.5, temperature 0 (calloc'd layers). */
int jdo_own_alloc(jdo_own *m, const jdo_config *c) {
    memset(m, 0, sizeof(*m));
    m->c = *c;
    int D = c->dim, qd = c->n_heads * c->head_dim, kd = c->n_kv_heads * c->head_dim, H = c->hidden_dim, V = c->vocab_size;
    if (c->depth < 1 || c->depth > JDO_MAX_LAYERS || c->initial_experts > JDO_MAX_EXPERTS) return -1;
    m->tok_emb = calloc((size_t)V * D, 4); m->output = calloc((size_t)V * D, 4); m->output_norm = malloc((size_t)D * 4);
    if (!m->tok_emb || !m->output || !m->output_norm) return -1;
    for (int i = 0; i < D; i++) m->output_norm[i] = 1.0f;
    for (int l = 0; l < c->depth; l++) {
        jdo_layer *L = &m->layers[l];
        L->attn_norm = malloc((size_t)D * 4); L->ffn_norm = malloc((size_t)D * 4);
        for (int i = 0; i < D; i++) { L->attn_norm[i] = 1.0f; L->ffn_norm[i] = 1.0f; }
        L->wq = calloc((size_t)qd * D, 4); L->wk = calloc((size_t)kd * D, 4); L->wv = calloc((size_t)kd * D, 4);
        L->wo = calloc((size_t)D * qd, 4); L->w_vote = calloc((size_t)JDO_MAX_EXPERTS * D, 4);
        L->consensus = 0.5f; L->temperature = 0.0f;
        for (int e = 0; e < c->initial_experts; e++) {
            L->w_gate[e] = calloc((size_t)H * D, 4); L->w_up[e] = calloc((size_t)H * D, 4); L->w_down[e] = calloc((size_t)D * H, 4);
            if (!L->w_gate[e] || !L->w_up[e] || !L->w_down[e]) return -1;
            L->alive[e] = 1;
        }
        if (!L->wq || !L->wk || !L->wv || !L->wo || !L->w_vote) return -1;
    }
    return 0;
}

static void jdo_fill(float *p, size_t n, uint64_t *s, float std) { for (size_t i = 0; i < n; i++) p[i] = jdo_rand_normal(s) * std; }

/* Synthetic seeded weights.  State = splitmix64(seed); every tensor is overwritten with
 * rand_normal()*std in this order: tok_emb, output, then per layer wq, wk, wv, wo,
 * w_vote (all 16 rows), then experts e = 0..initial-1 as gate, up, down.  Norms stay 1.
 * With draw_masks, the same stream then draws per layer a target alive count in
 * [max(2, n-3), n] and kills uniformly drawn slots until the target is reached. */
void jdo_own_fill_seeded(jdo_own *m, uint64_t seed, float std, int draw_masks) {
    const jdo_config *c = &m->c;
    int D = c->dim, qd = c->n_heads * c->head_dim, kd = c->n_kv_heads * c->head_dim, H = c->hidden_dim, V = c->vocab_size;
    uint64_t s = jdo_splitmix64(seed);
    jdo_fill(m->tok_emb, (size_t)V * D, &s, std);
    jdo_fill(m->output, (size_t)V * D, &s, std);
    for (int l = 0; l < c->depth; l++) {
        jdo_layer *L = &m->layers[l];
        jdo_fill(L->wq, (size_t)qd * D, &s, std); jdo_fill(L->wk, (size_t)kd * D, &s, std);
        jdo_fill(L->wv, (size_t)kd * D, &s, std); jdo_fill(L->wo, (size_t)D * qd, &s, std);
        jdo_fill(L->w_vote, (size_t)JDO_MAX_EXPERTS * D, &s, std);
        for (int e = 0; e < c->initial_experts; e++) {
            jdo_fill(L->w_gate[e], (size_t)H * D, &s, std); jdo_fill(L->w_up[e], (size_t)H * D, &s, std);
            jdo_fill(L->w_down[e], (size_t)D * H, &s, std);
        }
    }
    if (draw_masks) {
        int n0 = c->initial_experts;
        int lo = n0 - 3 < JDO_MIN_EXPERTS ? JDO_MIN_EXPERTS : n0 - 3;
        for (int l = 0; l < c->depth; l++) {
            jdo_layer *L = &m->layers[l];
            int target = lo + (int)(jdo_rng_next(&s) % (uint64_t)(n0 - lo + 1));
            int n = n0;
            while (n > target) { int e = (int)(jdo_rng_next(&s) % (uint64_t)n0); if (L->alive[e]) { L->alive[e] = 0; n--; } }
        }
    }
}

void jdo_own_free(jdo_own *m) {
    free(m->tok_emb); free(m->output); free(m->output_norm);
    for (int l = 0; l < JDO_MAX_LAYERS; l++) {
        jdo_layer *L = &m->layers[l];
        free(L->attn_norm); free(L->ffn_norm); free(L->wq); free(L->wk); free(L->wv); free(L->wo); free(L->w_vote);
        for (int e = 0; e < JDO_MAX_EXPERTS; e++) { free(L->w_gate[e]); free(L->w_up[e]); free(L->w_down[e]); }
    }
    memset(m, 0, sizeof(*m));
}

/* janusdoe.c:853-877 alloc_run: scratch, KV [depth][seq_len][kd], RoPE cache */
int jdo_own_state_alloc(const jdo_own *m, jdo_own_state *s) {
    const jdo_config *c = &m->c;
    memset(s, 0, sizeof(*s));
    int kd = c->n_kv_heads * c->head_dim, half = c->head_dim / 2;
    s->x = calloc(c->dim, 4); s->xb = calloc(c->dim, 4); s->xb2 = calloc(c->dim, 4);
    s->hb = calloc(c->hidden_dim, 4); s->hb2 = calloc(c->hidden_dim, 4);
    s->q = calloc((size_t)c->n_heads * c->head_dim, 4); s->k = calloc(kd, 4); s->v = calloc(kd, 4);
    s->att = calloc((size_t)c->n_heads * c->seq_len, 4); s->logits = calloc(c->vocab_size, 4);
    s->key_cache = calloc((size_t)c->depth * c->seq_len * kd, 4);
    s->value_cache = calloc((size_t)c->depth * c->seq_len * kd, 4);
    s->cos_cache = calloc((size_t)c->seq_len * half, 4); s->sin_cache = calloc((size_t)c->seq_len * half, 4);
    s->expert_out = calloc(c->dim, 4);
    if (!s->key_cache || !s->value_cache || !s->cos_cache) return -1;
    for (int p = 0; p < c->seq_len; p++)
        for (int i = 0; i < half; i++) {
            float freq = 1.0f / powf(c->rope_theta, (float)(2 * i) / (float)c->head_dim);
            float ang = (float)p * freq;
            s->cos_cache[p * half + i] = cosf(ang);
            s->sin_cache[p * half + i] = sinf(ang);
        }
    jdo_own_state_reset(m, s);
    return 0;
}
/* Fresh sequence: zero KV (janusdoe.c:3656-3657) and restart every layer's EMA. */
void jdo_own_state_reset(const jdo_own *m, jdo_own_state *s) {
    const jdo_config *c = &m->c;
    size_t n = (size_t)c->depth * c->seq_len * c->n_kv_heads * c->head_dim;
    memset(s->key_cache, 0, n * 4); memset(s->value_cache, 0, n * 4);
    for (int l = 0; l < JDO_MAX_LAYERS; l++) s->consensus[l] = l < c->depth ? m->layers[l].consensus : 0.5f;
}
void jdo_own_state_free(jdo_own_state *s) {
    free(s->x); free(s->xb); free(s->xb2); free(s->hb); free(s->hb2); free(s->q); free(s->k); free(s->v);
    free(s->att); free(s->logits); free(s->key_cache); free(s->value_cache); free(s->cos_cache); free(s->sin_cache);
    free(s->expert_out); memset(s, 0, sizeof(*s));
}

/* janusdoe.c:779-838 parliament_elect.  The harmonic term 0.1*expert_resonance() is
 * exactly 0 during decode: RunState.hs is zeroed by alloc_run (janusdoe.c:875) and
 * forward_token never writes it, so every amplitude is 0 (janusdoe.c:690-701). */
int jdo_parliament_elect(const jdo_layer *lw, float *consensus_io, const float *in, int dim,
                         int *selected, float *weights, jdo_elect *tr) {
    int n_alive = 0, alive_idx[JDO_MAX_EXPERTS];
    for (int e = 0; e < JDO_MAX_EXPERTS; e++) if (lw->alive[e]) alive_idx[n_alive++] = e;
    if (tr) { memset(tr, 0, sizeof(*tr)); tr->n_alive = n_alive; }
    if (n_alive < JDO_MIN_EXPERTS) { if (tr) tr->ema = *consensus_io; return 0; }
    float votes[JDO_MAX_EXPERTS];
    for (int i = 0; i < n_alive; i++) {
        int e = alive_idx[i];
        const float *row = lw->w_vote + (size_t)e * dim;
        float dot = 0; for (int j = 0; j < dim; j++) dot += row[j] * in[j];
        float res = 0.0f;
        votes[e] = dot + 0.1f * res;
    }
    float mean_v = 0; for (int i = 0; i < n_alive; i++) mean_v += votes[alive_idx[i]];
    mean_v /= n_alive;
    float var_v = 0; for (int i = 0; i < n_alive; i++) { float d = votes[alive_idx[i]] - mean_v; var_v += d * d; }
    var_v /= n_alive;
    float std_v = sqrtf(var_v + 1e-8f);
    float cons = fminf(1.0f, std_v / (fabsf(mean_v) + 1.0f));
    *consensus_io = 0.9f * *consensus_io + 0.1f * cons;
    int k = (int)(n_alive * (1.0f - *consensus_io));
    if (k < 2) k = 2;
    if (k > n_alive) k = n_alive;
    int used[JDO_MAX_EXPERTS] = {0};
    for (int ki = 0; ki < k; ki++) {
        float bv = -1e30f; int bi = 0;
        for (int i = 0; i < n_alive; i++) { int e = alive_idx[i]; if (!used[e] && votes[e] > bv) { bv = votes[e]; bi = e; } }
        selected[ki] = bi; weights[ki] = votes[bi]; used[bi] = 1;
    }
    float temp = (lw->temperature > 0.05f) ? lw->temperature : 1.0f;
    float mx = weights[0]; for (int i = 1; i < k; i++) if (weights[i] > mx) mx = weights[i];
    float sum = 0; for (int i = 0; i < k; i++) { weights[i] = expf((weights[i] - mx) / temp); sum += weights[i]; }
    for (int i = 0; i < k; i++) weights[i] /= sum;
    if (tr) {
        tr->k = k; tr->ema = *consensus_io;
        for (int i = 0; i < k; i++) { tr->sel[i] = selected[i]; tr->w[i] = weights[i]; }
        for (int i = 0; i < n_alive; i++) tr->votes[alive_idx[i]] = votes[alive_idx[i]];
    }
    return k;
}

/* janusdoe.c:879-934 forward_token, with the EMA state held per sequence. */
const float *jdo_own_forward(const jdo_own *m, jdo_own_state *s, int token, int pos, jdo_elect *trace) {
    const jdo_config *c = &m->c;
    int D = c->dim, kd = c->n_kv_heads * c->head_dim, hd = c->head_dim, H = c->hidden_dim;
    int hg = c->n_heads / c->n_kv_heads; float sc = 1.0f / sqrtf((float)hd);
    memcpy(s->x, m->tok_emb + (size_t)token * D, (size_t)D * 4);
    int adepth = (c->active_depth > 0 && c->active_depth <= c->depth) ? c->active_depth : c->depth;
    for (int l = 0; l < adepth; l++) {
        const jdo_layer *lw = &m->layers[l];
        jdo_rmsnorm(s->xb, s->x, lw->attn_norm, D, c->norm_eps);
        jdo_matvec(s->q, lw->wq, s->xb, c->n_heads * hd, D);
        jdo_matvec(s->k, lw->wk, s->xb, c->n_kv_heads * hd, D);
        jdo_matvec(s->v, lw->wv, s->xb, c->n_kv_heads * hd, D);
        for (int h = 0; h < c->n_heads; h++) jdo_rope_cache(s->q + h * hd, pos, s->cos_cache, s->sin_cache, hd);
        for (int h = 0; h < c->n_kv_heads; h++) jdo_rope_cache(s->k + h * hd, pos, s->cos_cache, s->sin_cache, hd);
        size_t co = (size_t)l * c->seq_len * kd + (size_t)pos * kd;
        memcpy(s->key_cache + co, s->k, (size_t)kd * 4);
        memcpy(s->value_cache + co, s->v, (size_t)kd * 4);
        for (int h = 0; h < c->n_heads; h++) {
            int kvh = h / hg; float *qh = s->q + h * hd; float *att = s->att + (size_t)h * c->seq_len;
            for (int t = 0; t <= pos; t++) {
                size_t ko = (size_t)l * c->seq_len * kd + (size_t)t * kd + (size_t)kvh * hd;
                float dot = 0; for (int d = 0; d < hd; d++) dot += qh[d] * s->key_cache[ko + d];
                att[t] = dot * sc;
            }
            if (c->attn_clamp > 0) { float inv = 1.0f / c->attn_clamp; for (int t = 0; t <= pos; t++) att[t] = c->attn_clamp * tanhf(att[t] * inv); }
            jdo_softmax(att, pos + 1);
            float *o = s->xb2 + h * hd; memset(o, 0, (size_t)hd * 4);
            for (int t = 0; t <= pos; t++) {
                float a = att[t]; size_t vo = (size_t)l * c->seq_len * kd + (size_t)t * kd + (size_t)kvh * hd;
                for (int d = 0; d < hd; d++) o[d] += a * s->value_cache[vo + d];
            }
        }
        jdo_matvec(s->xb, lw->wo, s->xb2, D, D);
        for (int i = 0; i < D; i++) s->x[i] += s->xb[i];
        jdo_rmsnorm(s->xb, s->x, lw->ffn_norm, D, c->norm_eps);
        memset(s->expert_out, 0, (size_t)D * 4);
        int selected[JDO_MAX_EXPERTS]; float weights[JDO_MAX_EXPERTS];
        int k = jdo_parliament_elect(lw, &s->consensus[l], s->xb, D, selected, weights, trace ? &trace[l] : NULL);
        for (int ki = 0; ki < k; ki++) {
            int e = selected[ki];
            jdo_matvec(s->hb, lw->w_gate[e], s->xb, H, D);
            jdo_matvec(s->hb2, lw->w_up[e], s->xb, H, D);
            for (int i = 0; i < H; i++) { float act = jdo_silu(s->hb[i]); s->hb[i] = act * s->hb2[i]; }
            jdo_matvec(s->xb2, lw->w_down[e], s->hb, D, H);
            for (int i = 0; i < D; i++) s->expert_out[i] += weights[ki] * s->xb2[i];
        }
        for (int i = 0; i < D; i++) s->x[i] += s->expert_out[i];
    }
    jdo_rmsnorm(s->x, s->x, m->output_norm, D, c->norm_eps);
    jdo_matvec(s->logits, m->output, s->x, c->vocab_size, D);
    return s->logits;
}

/* janusdoe.c:3637-3645 sample; the global rng_state becomes an explicit per-sequence state. */
int jdo_sample(float *logits, int V, float temp, int top_k, uint64_t *rng) {
    if (temp <= 0) { int b = 0; for (int i = 1; i < V; i++) if (logits[i] > logits[b]) b = i; return b; }
    for (int i = 0; i < V; i++) logits[i] /= temp;
    if (top_k > 0 && top_k < V) {
        float *s = malloc((size_t)V * 4); memcpy(s, logits, (size_t)V * 4);
        for (int i = 0; i < top_k; i++) { int b = i; for (int j = i + 1; j < V; j++) if (s[j] > s[b]) b = j; float t = s[i]; s[i] = s[b]; s[b] = t; }
        float th = s[top_k - 1]; free(s);
        for (int i = 0; i < V; i++) if (logits[i] < th) logits[i] = -1e30f;
    }
    jdo_softmax(logits, V);
    float r = jdo_rand_uniform(rng), cum = 0;
    for (int i = 0; i < V; i++) { cum += logits[i]; if (cum >= r) return i; }
    return V - 1;
}
/* janusdoe.c:3637 (temp <= 0 branch) and janusdoe.c:3374-3375: first index of the maximum */
int jdo_argmax(const float *lg, int V) { int b = 0; for (int i = 1; i < V; i++) if (lg[i] > lg[b]) b = i; return b; }

/* Synthetic prompt of sequence s: state = splitmix64(seed*1000+s); ids = rng_next() % V.
 * The state left afterwards is that sequence's sampling state. */
void jdo_prompt(uint64_t seq_seed, int V, int n, int *out, uint64_t *rng_after) {
    uint64_t s = jdo_splitmix64(seq_seed);
    for (int i = 0; i < n; i++) out[i] = (int)(jdo_rng_next(&s) % (uint64_t)V);
    if (rng_after) *rng_after = s;
}

/* ============================ packed quant ============================== */

/* janusdoe.c:2545-2553 jd_f16_to_f32: exact IEEE half -> float, subnormals included */
float jdo_f16_to_f32(uint16_t h) {
    uint32_t sign = (h >> 15) & 1, ex = (h >> 10) & 0x1F, mant = h & 0x3FF, f;
    if (ex == 0) {
        if (mant == 0) f = sign << 31;
        else { ex = 1; while (!(mant & 0x400)) { mant <<= 1; ex--; } mant &= 0x3FF; f = (sign << 31) | ((ex + 127 - 15) << 23) | (mant << 13); }
    } else if (ex == 31) f = (sign << 31) | 0x7F800000 | (mant << 13);
    else f = (sign << 31) | ((ex + 127 - 15) << 23) | (mant << 13);
    float r; memcpy(&r, &f, 4); return r;
}
static float jdo_h(const uint8_t *b) { return jdo_f16_to_f32((uint16_t)(b[0] | (b[1] << 8))); }
/* janusdoe.c:2559-2561 jd_smk4: 6-bit (scale, min) of sub-block j from the 12 packed bytes */
static void jdo_smk4(int j, const uint8_t *sc, uint8_t *s, uint8_t *m) {
    if (j < 4) { *s = sc[j] & 63; *m = sc[j + 4] & 63; }
    else { *s = (uint8_t)((sc[j + 4] & 0x0F) | ((sc[j - 4] >> 6) << 4)); *m = (uint8_t)((sc[j + 4] >> 4) | ((sc[j] >> 6) << 4)); }
}
/* janusdoe.c:2597-2601 jd_quant_bytes */
uint64_t jdo_quant_bytes(int dt, uint64_t n) {
    switch (dt) {
    case 0: return n * 4; case 1: return n * 2; case 2: return (n / 32) * 18;
    case 6: return (n / 32) * 22; case 8: return (n / 32) * 34;
    case 12: return (n / 256) * 144; case 14: return (n / 256) * 210; default: return 0;
    }
}
/* janusdoe.c:2563-2596, 2602-2610 jd_dequant_*: whole-tensor dequantisation */
int jdo_dequant(const uint8_t *src, float *out, uint64_t n, int dt) {
    if (dt == 0) { memcpy(out, src, n * 4); return 0; }
    if (dt == 1) { for (uint64_t i = 0; i < n; i++) out[i] = jdo_f16_to_f32((uint16_t)(src[2 * i] | (src[2 * i + 1] << 8))); return 0; }
    if (dt == 2) {
        for (uint64_t i = 0; i < n / 32; i++) { const uint8_t *b = src + i * 18; float d = jdo_h(b);
            for (int j = 0; j < 16; j++) { out[i * 32 + j] = (float)((b[2 + j] & 0x0F) - 8) * d; out[i * 32 + j + 16] = (float)((b[2 + j] >> 4) - 8) * d; } }
        return 0;
    }
    if (dt == 6) {
        for (uint64_t i = 0; i < n / 32; i++) { const uint8_t *b = src + i * 22; float d = jdo_h(b);
            uint32_t qh = b[2] | (b[3] << 8) | (b[4] << 16) | ((uint32_t)b[5] << 24); const uint8_t *qs = b + 6;
            for (int j = 0; j < 16; j++) { int lo = qs[j] & 0x0F, hi = qs[j] >> 4, h0 = (qh >> j) & 1, h1 = (qh >> (j + 16)) & 1;
                out[i * 32 + j] = (float)((lo | (h0 << 4)) - 16) * d; out[i * 32 + j + 16] = (float)((hi | (h1 << 4)) - 16) * d; } }
        return 0;
    }
    if (dt == 8) {
        for (uint64_t i = 0; i < n / 32; i++) { const uint8_t *b = src + i * 34; float d = jdo_h(b);
            for (int j = 0; j < 32; j++) out[i * 32 + j] = (float)((int8_t)b[2 + j]) * d; }
        return 0;
    }
    if (dt == 12) {
        for (uint64_t i = 0; i < n / 256; i++) { const uint8_t *b = src + i * 144; float d = jdo_h(b), dmin = jdo_h(b + 2);
            const uint8_t *sc = b + 4, *qs = b + 16; int is = 0, qi = 0; uint64_t oi = i * 256;
            for (int j = 0; j < 256; j += 64) { uint8_t s0, m0, s1, m1; jdo_smk4(is, sc, &s0, &m0); jdo_smk4(is + 1, sc, &s1, &m1);
                float d1 = d * s0, mm1 = dmin * m0, d2 = d * s1, mm2 = dmin * m1;
                for (int l = 0; l < 32; l++) out[oi + j + l] = d1 * (float)(qs[qi + l] & 0x0F) - mm1;
                for (int l = 0; l < 32; l++) out[oi + j + 32 + l] = d2 * (float)(qs[qi + l] >> 4) - mm2;
                qi += 32; is += 2; } }
        return 0;
    }
    if (dt == 14) {
        for (uint64_t i = 0; i < n / 256; i++) { const uint8_t *b = src + i * 210, *ql = b, *qh = b + 128, *sc = b + 192;
            float d = jdo_f16_to_f32((uint16_t)(b[208] | (b[209] << 8))); uint64_t oi = i * 256;
            for (int h = 0; h < 2; h++) { const uint8_t *qlp = ql + h * 64, *qhp = qh + h * 32, *scp = sc + h * 8; uint64_t yo = oi + h * 128;
                for (int l = 0; l < 32; l++) { int is = l / 16;
                    int q1 = (qlp[l] & 0x0F) | ((qhp[l] >> 0) & 3) << 4, q2 = (qlp[l + 32] & 0x0F) | ((qhp[l] >> 2) & 3) << 4;
                    int q3 = (qlp[l] >> 4) | ((qhp[l] >> 4) & 3) << 4, q4 = (qlp[l + 32] >> 4) | ((qhp[l] >> 6) & 3) << 4;
                    out[yo + l] = d * (float)((int8_t)scp[is]) * (float)(q1 - 32);
                    out[yo + l + 32] = d * (float)((int8_t)scp[is + 2]) * (float)(q2 - 32);
                    out[yo + l + 64] = d * (float)((int8_t)scp[is + 4]) * (float)(q3 - 32);
                    out[yo + l + 96] = d * (float)((int8_t)scp[is + 6]) * (float)(q4 - 32); } } }
        return 0;
    }
    return -1;
}
/* janusdoe.c:2630-2636 jd_pq_q8_0_rows: acc += (d*q)*x, one accumulator per row */
static void jdo_q8_0_rows(float *out, const uint8_t *W, const float *x, int r0, int r1, int c) {
    int nb = c / 32;
    for (int row = r0; row < r1; row++) { const uint8_t *rb = W + (size_t)row * nb * 34; float a = 0;
        for (int b = 0; b < nb; b++) { const uint8_t *bl = rb + (size_t)b * 34; float d = jdo_h(bl); const float *xb = x + (size_t)b * 32;
            for (int i = 0; i < 32; i++) a += d * (float)(int8_t)bl[2 + i] * xb[i]; }
        out[row] = a; }
}
/* janusdoe.c:2647-2659 jd_pq_q4_k_rows: acc += (d1*q - mm1)*x */
static void jdo_q4_k_rows(float *out, const uint8_t *W, const float *x, int r0, int r1, int c) {
    int nb = c / 256;
    for (int row = r0; row < r1; row++) { const uint8_t *rb = W + (size_t)row * nb * 144; float a = 0;
        for (int b = 0; b < nb; b++) { const uint8_t *bl = rb + (size_t)b * 144;
            float d = jdo_h(bl), dmin = jdo_h(bl + 2); const uint8_t *sc = bl + 4, *qs = bl + 16; const float *xb = x + (size_t)b * 256; int is = 0, qi = 0;
            for (int j = 0; j < 256; j += 64) { uint8_t s0, m0, s1, m1; jdo_smk4(is, sc, &s0, &m0); jdo_smk4(is + 1, sc, &s1, &m1);
                float d1 = d * s0, mm1 = dmin * m0, d2 = d * s1, mm2 = dmin * m1;
                for (int l = 0; l < 32; l++) a += (d1 * (float)(qs[qi + l] & 0x0F) - mm1) * xb[j + l];
                for (int l = 0; l < 32; l++) a += (d2 * (float)(qs[qi + l] >> 4) - mm2) * xb[j + 32 + l];
                qi += 32; is += 2; } }
        out[row] = a; }
}
/* janusdoe.c:2619-2623 jd_pq_f16_rows */
static void jdo_f16_rows(float *out, const uint8_t *W, const float *x, int r0, int r1, int c) {
    const uint16_t *Wh = (const uint16_t *)W;
    for (int row = r0; row < r1; row++) { const uint16_t *r = Wh + (size_t)row * c; float a = 0; for (int j = 0; j < c; j++) a += jdo_f16_to_f32(r[j]) * x[j]; out[row] = a; }
}
/* janusdoe.c:2624-2629 jd_pq_q4_0_rows */
static void jdo_q4_0_rows(float *out, const uint8_t *W, const float *x, int r0, int r1, int c) {
    int nb = c / 32;
    for (int row = r0; row < r1; row++) { const uint8_t *rb = W + (size_t)row * nb * 18; float a = 0;
        for (int b = 0; b < nb; b++) { const uint8_t *bl = rb + (size_t)b * 18; float d = jdo_h(bl); const float *xb = x + (size_t)b * 32;
            for (int i = 0; i < 16; i++) { int lo = (int)(bl[2 + i] & 0x0F) - 8, hi = (int)(bl[2 + i] >> 4) - 8; a += d * lo * xb[i]; a += d * hi * xb[i + 16]; } }
        out[row] = a; }
}
/* janusdoe.c:2637-2646 jd_pq_q5_0_rows */
static void jdo_q5_0_rows(float *out, const uint8_t *W, const float *x, int r0, int r1, int c) {
    int nb = c / 32;
    for (int row = r0; row < r1; row++) { const uint8_t *rb = W + (size_t)row * nb * 22; float a = 0;
        for (int b = 0; b < nb; b++) { const uint8_t *bl = rb + (size_t)b * 22; float d = jdo_h(bl);
            uint32_t qh = (uint32_t)bl[2] | ((uint32_t)bl[3] << 8) | ((uint32_t)bl[4] << 16) | ((uint32_t)bl[5] << 24);
            const uint8_t *qs = bl + 6; const float *xb = x + (size_t)b * 32;
            for (int j = 0; j < 16; j++) { int lo = qs[j] & 0x0F, hi = qs[j] >> 4, h0 = (qh >> j) & 1, h1 = (qh >> (j + 16)) & 1;
                a += d * (float)((lo | (h0 << 4)) - 16) * xb[j]; a += d * (float)((hi | (h1 << 4)) - 16) * xb[j + 16]; } }
        out[row] = a; }
}
/* janusdoe.c:2660-2673 jd_pq_q6_k_rows */
static void jdo_q6_k_rows(float *out, const uint8_t *W, const float *x, int r0, int r1, int c) {
    int nb = c / 256;
    for (int row = r0; row < r1; row++) { const uint8_t *rb = W + (size_t)row * nb * 210; float a = 0;
        for (int b = 0; b < nb; b++) { const uint8_t *bl = rb + (size_t)b * 210, *ql = bl, *qh = bl + 128;
            const int8_t *sc = (const int8_t *)(bl + 192); float d = jdo_f16_to_f32((uint16_t)(bl[208] | (bl[209] << 8)));
            const float *xb = x + (size_t)b * 256;
            for (int n = 0; n < 256; n += 128) { const uint8_t *qlh = ql + (n / 128) * 64, *qhh = qh + (n / 128) * 32; const int8_t *sch = sc + (n / 128) * 8;
                for (int l = 0; l < 32; l++) { int is = l / 16;
                    int q1 = (int)((qlh[l] & 0x0F) | (((qhh[l] >> 0) & 3) << 4)) - 32, q2 = (int)((qlh[l + 32] & 0x0F) | (((qhh[l] >> 2) & 3) << 4)) - 32;
                    int q3 = (int)((qlh[l] >> 4) | (((qhh[l] >> 4) & 3) << 4)) - 32, q4 = (int)((qlh[l + 32] >> 4) | (((qhh[l] >> 6) & 3) << 4)) - 32;
                    a += d * sch[is + 0] * q1 * xb[n + l]; a += d * sch[is + 2] * q2 * xb[n + l + 32];
                    a += d * sch[is + 4] * q3 * xb[n + l + 64]; a += d * sch[is + 6] * q4 * xb[n + l + 96]; } } }
        out[row] = a; }
}
/* janusdoe.c:2674-2680 jd_pq_for + janusdoe.c:2685-2694 jd_qmatvec: 0 ok, -1 unsupported */
int jdo_qmatvec(float *out, const uint8_t *W, int dt, const float *x, int r, int c) {
    jdo_rows_fn fn = NULL;
    switch (dt) {
    case 1: fn = jdo_f16_rows; break;
    case 2: fn = (c % 32) ? NULL : jdo_q4_0_rows; break;
    case 6: fn = (c % 32) ? NULL : jdo_q5_0_rows; break;
    case 8: fn = (c % 32) ? NULL : jdo_q8_0_rows; break;
    case 12: fn = (c % 256) ? NULL : jdo_q4_k_rows; break;
    case 14: fn = (c % 256) ? NULL : jdo_q6_k_rows; break;
    }
    if (!fn) return -1;
    jdo_run_rows(fn, out, W, x, r, c);
    return 0;
}
/* janusdoe.c:2733-2743 jd_mv: packed -> jd_qmatvec (abort on failure), f32 -> matvec */
static void jdo_mv(float *out, const void *W, int dt, const float *x, int r, int c) {
    if (dt) {
        if (jdo_qmatvec(out, (const uint8_t *)W, dt, x, r, c) == 0) return;
        fprintf(stderr, "oracle: packed dtype %d unsupported (r=%d c=%d)\n", dt, r, c); abort();
    }
    jdo_matvec(out, (const float *)W, x, r, c);
}

/* ============================ host GGUF ================================= */

/* janusdoe.c:3153-3156 arch_rope_norm */
int jdo_rope_norm_for_arch(const char *arch) {
    return strcmp(arch, "llama") == 0 || strcmp(arch, "mistral") == 0 || strcmp(arch, "mistral3") == 0 || strcmp(arch, "mistral4") == 0;
}

static int jdo_rows_ok(int dt, int c) {
    switch (dt) { case 1: return 1; case 2: case 6: case 8: return c % 32 == 0; case 12: case 14: return c % 256 == 0; }
    return 0;
}
/* janusdoe.c:2817-2833 jd_host_resolve: f32 points into the map; a supported packed matvec
 * weight stays packed; tok_emb/norms and unsupported dtypes are dequantised once. */
static void *jdo_resolve(jdo_host *h, const uint8_t *raw, const uint8_t *pend, int dt, uint64_t ne, int c, int want_f32, int *out_dt) {
    *out_dt = 0;
    uint64_t bytes = jdo_quant_bytes(dt, ne);
    if (dt != 0 && bytes == 0) return NULL;
    if (bytes == 0) bytes = ne * 4;
    if (raw + bytes > pend) return NULL;
    if (dt == 0) return (void *)raw;
    if (!want_f32 && jdo_rows_ok(dt, c)) { *out_dt = dt; return (void *)raw; }
    float *buf = malloc(ne * 4); if (!buf) return NULL;
    if (jdo_dequant(raw, buf, ne, dt) != 0) { free(buf); return NULL; }
    if (h->n_dq < (int)(sizeof(h->dq) / sizeof(h->dq[0]))) h->dq[h->n_dq++] = buf; else { free(buf); return NULL; }
    return buf;
}

/* janusdoe.c:2837-3048 gguf_host_load, decode-relevant parts: header, key/value scan with
 * the same substring matching and defaults, tensor table, 32-byte data alignment, tensor
 * resolution, tied output, essential-weight and standard-FFN checks.  The LoRA parliament
 * starts empty here; jdo_host_lora_seed fills it.  Returns 1 on success, 0 on failure. */
int jdo_host_load(jdo_host *h, const char *path, int rope_override, int lora_rank) {
    memset(h, 0, sizeof(*h));
    h->bos = h->eos = -1; h->lora_alpha = 0.1f; h->lora_rank = lora_rank;
    int fd = open(path, O_RDONLY); if (fd < 0) return 0;
    struct stat st; if (fstat(fd, &st) != 0) { close(fd); return 0; }
    h->map_size = (size_t)st.st_size;
    void *mp = mmap(NULL, h->map_size, PROT_READ, MAP_PRIVATE, fd, 0); close(fd);
    if (mp == MAP_FAILED) return 0;
    h->map = (uint8_t *)mp;
    const uint8_t *p = h->map, *pend = h->map + h->map_size;
    struct { char name[96]; uint32_t ndim; uint64_t dims[4]; uint32_t dtype; uint64_t off; } *ti = NULL;
#define NEED(n) do { if ((uint64_t)(pend - p) < (uint64_t)(n)) goto bail; } while (0)
#define RD(T, v) T v; NEED(sizeof(T)); memcpy(&v, p, sizeof(T)); p += sizeof(T)
    { RD(uint32_t, magic); if (magic != 0x46554747) goto bail; }
    { RD(uint32_t, ver); (void)ver; }
    RD(uint64_t, n_tensors);
    RD(uint64_t, n_kv);
    for (uint64_t i = 0; i < n_kv; i++) {
        RD(uint64_t, klen);
        char key[256];
        NEED(klen);
        if (klen > 255) { key[0] = 0; } else { memcpy(key, p, klen); key[klen] = 0; }
        p += klen;
        RD(uint32_t, vt);
        if (vt == 8) {
            RD(uint64_t, vlen); NEED(vlen);
            if (strstr(key, "general.architecture") && vlen < 64) { memcpy(h->arch, p, vlen); h->arch[vlen] = 0; }
            p += vlen;
        } else if (vt == 4) {
            RD(uint32_t, v);
            if (strstr(key, "embedding_length")) h->dim = (int)v;
            else if (strstr(key, "block_count")) h->n_layers = (int)v;
            else if (strstr(key, "head_count") && !strstr(key, "kv")) h->n_heads = (int)v;
            else if (strstr(key, "head_count_kv")) h->n_kv_heads = (int)v;
            else if (strstr(key, "feed_forward_length")) h->hidden = (int)v;
            else if (strstr(key, "vocab_size")) h->vocab = (int)v;
            else if (strstr(key, "attention.key_length")) h->head_dim = (int)v;
            else if (strstr(key, "bos_token_id")) h->bos = (int)v;
            else if (strstr(key, "eos_token_id")) h->eos = (int)v;
        } else if (vt == 6) {
            RD(float, fv);
            if (strstr(key, "rope.freq_base")) h->rope_theta = fv;
            else if (strstr(key, "rms_epsilon")) h->rms_eps = fv;
        } else if (vt == 0 || vt == 1 || vt == 7) { NEED(1); p += 1; }
        else if (vt == 2 || vt == 3) { NEED(2); p += 2; }
        else if (vt == 5) { NEED(4); p += 4; }
        else if (vt == 10 || vt == 11 || vt == 12) { NEED(8); p += 8; }
        else if (vt == 9) {
            RD(uint32_t, at); RD(uint64_t, alen);
            if (at == 8) {
                for (uint64_t a = 0; a < alen; a++) { RD(uint64_t, sl); if (sl > 1000000) goto bail; NEED(sl); p += sl; }
            } else {
                uint64_t esz = (at == 0 || at == 1 || at == 7) ? 1 : (at == 2 || at == 3) ? 2 : (at == 4 || at == 5 || at == 6) ? 4 : (at == 10 || at == 11 || at == 12) ? 8 : 0;
                if (esz == 0) goto bail;
                NEED(alen * esz); p += alen * esz;
            }
        } else { NEED(4); p += 4; }
    }
    if (h->dim == 0 || h->dim > 16384 || h->n_layers == 0) goto bail;
    if (h->n_heads == 0) h->n_heads = h->dim / 64;
    if (h->n_kv_heads == 0) h->n_kv_heads = h->n_heads;
    if (h->head_dim == 0) h->head_dim = h->dim / h->n_heads;
    if (h->hidden == 0) h->hidden = h->dim * 4;
    if (h->rope_theta == 0.0f) h->rope_theta = 10000.0f;
    if (h->rms_eps == 0.0f) h->rms_eps = 1e-6f;
    if (n_tensors > 10000) goto bail;
    ti = calloc(n_tensors ? n_tensors : 1, sizeof(*ti)); if (!ti) goto bail;
    for (uint64_t i = 0; i < n_tensors; i++) {
        RD(uint64_t, nlen); if (nlen > 256) goto bail;
        int nl = nlen < 95 ? (int)nlen : 95;
        NEED(nlen); memcpy(ti[i].name, p, nl); ti[i].name[nl] = 0; p += nlen;
        { RD(uint32_t, nd); ti[i].ndim = nd; }
        if (ti[i].ndim > 4) goto bail;
        for (uint32_t d = 0; d < ti[i].ndim; d++) { RD(uint64_t, dv); ti[i].dims[d] = dv; }
        { RD(uint32_t, dt); ti[i].dtype = dt; }
        { RD(uint64_t, of); ti[i].off = of; }
    }
    {
        uint64_t hdr = (uint64_t)(p - h->map), data_start = ((hdr + 31) / 32) * 32;
        for (uint64_t i = 0; i < n_tensors; i++) {
            int dt = (int)ti[i].dtype, wdt = 0;
            if (data_start + ti[i].off > h->map_size) continue;   /* resolve() rejects it */
            const uint8_t *raw = h->map + data_start + ti[i].off;
            uint64_t ne = 1; for (uint32_t d = 0; d < ti[i].ndim; d++) ne *= ti[i].dims[d];
            int c = ti[i].ndim > 0 ? (int)ti[i].dims[0] : 0;
            const char *n = ti[i].name;
            if (strcmp(n, "token_embd.weight") == 0) {
                h->tok_emb = jdo_resolve(h, raw, pend, dt, ne, c, 1, &wdt);
                if (h->vocab == 0) h->vocab = (int)ti[i].dims[1];
            } else if (strcmp(n, "output_norm.weight") == 0) h->output_norm = jdo_resolve(h, raw, pend, dt, ne, c, 1, &wdt);
            else if (strcmp(n, "output.weight") == 0) h->output = jdo_resolve(h, raw, pend, dt, ne, c, 0, &h->output_dt);
            else {
                int l = -1; sscanf(n, "blk.%d.", &l);
                if (l >= 0 && l < JDO_MAX_LAYERS && l < h->n_layers) {
                    if (strstr(n, "attn_q.weight")) h->layers[l].wq = jdo_resolve(h, raw, pend, dt, ne, c, 0, &h->layers[l].wq_dt);
                    else if (strstr(n, "attn_k.weight")) h->layers[l].wk = jdo_resolve(h, raw, pend, dt, ne, c, 0, &h->layers[l].wk_dt);
                    else if (strstr(n, "attn_v.weight")) h->layers[l].wv = jdo_resolve(h, raw, pend, dt, ne, c, 0, &h->layers[l].wv_dt);
                    else if (strstr(n, "attn_output.weight")) h->layers[l].wo = jdo_resolve(h, raw, pend, dt, ne, c, 0, &h->layers[l].wo_dt);
                    else if (strstr(n, "ffn_gate.weight") && !strstr(n, "ffn_gate_inp")) h->layers[l].gate = jdo_resolve(h, raw, pend, dt, ne, c, 0, &h->layers[l].gate_dt);
                    else if (strstr(n, "ffn_up.weight")) h->layers[l].up = jdo_resolve(h, raw, pend, dt, ne, c, 0, &h->layers[l].up_dt);
                    else if (strstr(n, "ffn_down.weight")) h->layers[l].down = jdo_resolve(h, raw, pend, dt, ne, c, 0, &h->layers[l].down_dt);
                    else if (strstr(n, "attn_norm.weight")) h->layers[l].attn_norm = jdo_resolve(h, raw, pend, dt, ne, c, 1, &wdt);
                    else if (strstr(n, "ffn_norm.weight")) h->layers[l].ffn_norm = jdo_resolve(h, raw, pend, dt, ne, c, 1, &wdt);
                }
            }
        }
    }
    free(ti); ti = NULL;
    if (!h->output && h->tok_emb) { h->output = h->tok_emb; h->output_dt = 0; }
    if (!h->tok_emb || !h->output || !h->output_norm) goto bail;
    {
        int has_ffn = 0;
        for (int l = 0; l < h->n_layers && l < JDO_MAX_LAYERS; l++) if (h->layers[l].gate && h->layers[l].up && h->layers[l].down) has_ffn = 1;
        if (!has_ffn) goto bail;
    }
    h->rope_norm = rope_override >= 0 ? rope_override : jdo_rope_norm_for_arch(h->arch);
    for (int l = 0; l < h->n_layers && l < JDO_MAX_LAYERS; l++) {
        h->w_vote[l] = calloc((size_t)JDO_MAX_EXPERTS * h->dim, 4);
        if (!h->w_vote[l]) goto bail;
        h->consensus0[l] = 0.5f; h->attention_bias[l] = 0.0f; h->layer_focus[l] = 1.0f;
    }
#undef NEED
#undef RD
    return 1;
bail:
    free(ti);
    jdo_host_free(h);
    return 0;
}

/* Synthetic LoRA parliament: state = splitmix64(seed); per layer, the 16 vote rows are
 * drawn uniform in [-vote_amp, vote_amp) as (2u-1)*amp, then experts e < n_alive draw
 * A [D][r] and B [r][D] as rand_normal()*ab_std.  Experts >= n_alive are dead. */
void jdo_host_lora_seed(jdo_host *h, uint64_t seed, int n_alive, float ab_std, float vote_amp) {
    uint64_t s = jdo_splitmix64(seed);
    int D = h->dim, R = h->lora_rank;
    for (int l = 0; l < h->n_layers && l < JDO_MAX_LAYERS; l++) {
        for (int i = 0; i < JDO_MAX_EXPERTS * D; i++) h->w_vote[l][i] = (2.0f * jdo_rand_uniform(&s) - 1.0f) * vote_amp;
        for (int e = 0; e < JDO_MAX_EXPERTS; e++) {
            if (e < n_alive) {
                if (!h->A[l][e]) h->A[l][e] = calloc((size_t)D * R, 4);
                if (!h->B[l][e]) h->B[l][e] = calloc((size_t)R * D, 4);
                for (int j = 0; j < D * R; j++) h->A[l][e][j] = jdo_rand_normal(&s) * ab_std;
                for (int j = 0; j < R * D; j++) h->B[l][e][j] = jdo_rand_normal(&s) * ab_std;
                h->alive[l][e] = 1;
            } else h->alive[l][e] = 0;
        }
    }
}

void jdo_host_free(jdo_host *h) {
    for (int i = 0; i < h->n_dq; i++) free(h->dq[i]);
    if (h->map) munmap(h->map, h->map_size);
    for (int l = 0; l < JDO_MAX_LAYERS; l++) {
        free(h->w_vote[l]);
        for (int e = 0; e < JDO_MAX_EXPERTS; e++) { free(h->A[l][e]); free(h->B[l][e]); }
    }
    memset(h, 0, sizeof(*h));
}

int jdo_host_state_alloc(const jdo_host *h, jdo_host_state *s, int max_seq) {
    size_t n = (size_t)h->n_layers * max_seq * h->n_kv_heads * h->head_dim;
    memset(s, 0, sizeof(*s));
    s->max_seq = max_seq; s->kc = calloc(n, 4); s->vc = calloc(n, 4);
    s->host_x = calloc(h->dim, 4); s->host_dy = calloc(h->dim, 4);
    if (!s->kc || !s->vc || !s->host_x || !s->host_dy) return -1;
    jdo_host_state_reset(h, s);
    return 0;
}
void jdo_host_state_reset(const jdo_host *h, jdo_host_state *s) {
    size_t n = (size_t)h->n_layers * s->max_seq * h->n_kv_heads * h->head_dim;
    memset(s->kc, 0, n * 4); memset(s->vc, 0, n * 4);
    for (int l = 0; l < JDO_MAX_LAYERS; l++) s->consensus[l] = h->consensus0[l];
}
void jdo_host_state_free(jdo_host_state *s) {
    free(s->kc); free(s->vc); free(s->host_x); free(s->host_dy); memset(s, 0, sizeof(*s));
}

/* janusdoe.c:3054-3087 host_parliament_elect */
int jdo_host_elect(const jdo_host *h, int l, float *cons_io, const float *xn, int D, int *selected, float *weights, jdo_elect *tr) {
    int alive_idx[JDO_MAX_EXPERTS], na = 0;
    for (int e = 0; e < JDO_MAX_EXPERTS; e++) if (h->alive[l][e]) alive_idx[na++] = e;
    if (tr) { memset(tr, 0, sizeof(*tr)); tr->n_alive = na; tr->ema = *cons_io; }
    if (na == 0) return 0;
    if (na == 1) { selected[0] = alive_idx[0]; weights[0] = 1.0f; if (tr) { tr->k = 1; tr->sel[0] = alive_idx[0]; tr->w[0] = 1.0f; } return 1; }
    float votes[JDO_MAX_EXPERTS];
    for (int i = 0; i < na; i++) {
        int e = alive_idx[i]; const float *row = h->w_vote[l] + (size_t)e * D;
        float d = 0; for (int j = 0; j < D; j++) d += row[j] * xn[j];
        votes[e] = isfinite(d) ? d : -1e30f;
    }
    float mean = 0; for (int i = 0; i < na; i++) mean += votes[alive_idx[i]]; mean /= na;
    float var = 0; for (int i = 0; i < na; i++) { float dd = votes[alive_idx[i]] - mean; var += dd * dd; } var /= na;
    float cons = fminf(1.0f, sqrtf(var + 1e-8f) / (fabsf(mean) + 1.0f));
    *cons_io = 0.9f * *cons_io + 0.1f * cons;
    int k = (int)(na * (1.0f - *cons_io));
    if (k < 2) k = 2;
    if (k > na) k = na;
    int used[JDO_MAX_EXPERTS] = {0};
    for (int ki = 0; ki < k; ki++) {
        float bv = -1e30f; int bi = -1;
        for (int i = 0; i < na; i++) { int e = alive_idx[i]; if (!used[e] && votes[e] > bv) { bv = votes[e]; bi = e; } }
        if (bi < 0) for (int i = 0; i < na; i++) { int e = alive_idx[i]; if (!used[e]) { bi = e; break; } }
        selected[ki] = bi; weights[ki] = votes[bi]; used[bi] = 1;
    }
    float mx = weights[0]; for (int i = 1; i < k; i++) if (weights[i] > mx) mx = weights[i];
    float sum = 0; for (int i = 0; i < k; i++) { weights[i] = expf(weights[i] - mx); sum += weights[i]; }
    if (sum > 0.0f && isfinite(sum)) { for (int i = 0; i < k; i++) weights[i] /= sum; }
    else { for (int i = 0; i < k; i++) weights[i] = 1.0f / k; }
    if (tr) {
        tr->k = k; tr->ema = *cons_io;
        for (int i = 0; i < k; i++) { tr->sel[i] = selected[i]; tr->w[i] = weights[i]; }
        for (int i = 0; i < na; i++) tr->votes[alive_idx[i]] = votes[alive_idx[i]];
    }
    return k;
}

/* janusdoe.c:3160-3322 gguf_host_forward (the learning captures host_x/host_dy are not
 * part of the output and are left out). */
void jdo_host_forward(const jdo_host *h, jdo_host_state *s, int token, int pos, float *logits, jdo_elect *trace) {
    int D = h->dim, Hn = h->n_heads, HD = h->head_dim, KVH = h->n_kv_heads, HG = Hn / KVH;
    int qd = Hn * HD, kd = KVH * HD, HH = h->hidden, R = h->lora_rank, max_seq = s->max_seq;
    float *x = calloc(D, 4), *t = calloc(R > 0 ? R : 1, 4), *xn = calloc(D, 4), *q = calloc(qd, 4), *k = calloc(kd, 4), *v = calloc(kd, 4);
    float *ao_in = calloc(qd, 4), *ao = calloc(D, 4), *fn = calloc(D, 4), *gate = calloc(HH, 4), *up = calloc(HH, 4), *fo = calloc(D, 4);
    float *att = calloc((size_t)pos + 1, 4);
    if (token < h->vocab) memcpy(x, h->tok_emb + (size_t)token * D, (size_t)D * 4);
    for (int l = 0; l < h->n_layers && l < JDO_MAX_LAYERS; l++) {
        if (!h->layers[l].wq) continue;
        float ss = 0; for (int i = 0; i < D; i++) ss += x[i] * x[i];
        ss = 1.0f / sqrtf(ss / D + h->rms_eps);
        if (h->layers[l].attn_norm) for (int i = 0; i < D; i++) xn[i] = x[i] * ss * h->layers[l].attn_norm[i];
        else for (int i = 0; i < D; i++) xn[i] = x[i] * ss;
        jdo_mv(q, h->layers[l].wq, h->layers[l].wq_dt, xn, qd, D);
        jdo_mv(k, h->layers[l].wk, h->layers[l].wk_dt, xn, kd, D);
        jdo_mv(v, h->layers[l].wv, h->layers[l].wv_dt, xn, kd, D);
        int rn = h->rope_norm;
        for (int hh = 0; hh < Hn; hh++) {
            float *qh = q + hh * HD; int half = HD / 2;
            for (int i = 0; i < half; i++) {
                float ang = (float)pos / powf(h->rope_theta, 2.0f * i / (float)HD);
                float co = cosf(ang), si = sinf(ang);
                int a = rn ? 2 * i : i, b = rn ? 2 * i + 1 : i + half;
                float x0 = qh[a], x1 = qh[b];
                qh[a] = x0 * co - x1 * si; qh[b] = x0 * si + x1 * co;
            }
        }
        for (int hh = 0; hh < KVH; hh++) {
            float *kh = k + hh * HD; int half = HD / 2;
            for (int i = 0; i < half; i++) {
                float ang = (float)pos / powf(h->rope_theta, 2.0f * i / (float)HD);
                float co = cosf(ang), si = sinf(ang);
                int a = rn ? 2 * i : i, b = rn ? 2 * i + 1 : i + half;
                float x0 = kh[a], x1 = kh[b];
                kh[a] = x0 * co - x1 * si; kh[b] = x0 * si + x1 * co;
            }
        }
        size_t lo = (size_t)l * max_seq * kd;
        memcpy(s->kc + lo + (size_t)pos * kd, k, (size_t)kd * 4);
        memcpy(s->vc + lo + (size_t)pos * kd, v, (size_t)kd * 4);
        float bias = 1.0f + h->attention_bias[l];
        float sc = 1.0f / sqrtf((float)HD);
        memset(ao_in, 0, (size_t)qd * 4);
        for (int hh = 0; hh < Hn; hh++) {
            int kvh = hh / HG; float *qh = q + hh * HD;
            for (int tt = 0; tt <= pos; tt++) {
                const float *kt = s->kc + lo + (size_t)tt * kd + (size_t)kvh * HD;
                float d = 0; for (int i = 0; i < HD; i++) d += qh[i] * kt[i];
                att[tt] = d * sc * bias;
            }
            float mx = att[0]; for (int tt = 1; tt <= pos; tt++) if (att[tt] > mx) mx = att[tt];
            float se = 0; for (int tt = 0; tt <= pos; tt++) { att[tt] = expf(att[tt] - mx); se += att[tt]; }
            for (int tt = 0; tt <= pos; tt++) att[tt] /= se;
            float *oh = ao_in + hh * HD;
            for (int tt = 0; tt <= pos; tt++) {
                float a = att[tt]; const float *vt = s->vc + lo + (size_t)tt * kd + (size_t)kvh * HD;
                for (int i = 0; i < HD; i++) oh[i] += a * vt[i];
            }
        }
        memset(ao, 0, (size_t)D * 4);
        if (h->layers[l].wo) jdo_mv(ao, h->layers[l].wo, h->layers[l].wo_dt, ao_in, D, qd);
        for (int i = 0; i < D; i++) x[i] += ao[i];
        ss = 0; for (int i = 0; i < D; i++) ss += x[i] * x[i];
        ss = 1.0f / sqrtf(ss / D + h->rms_eps);
        if (h->layers[l].ffn_norm) for (int i = 0; i < D; i++) fn[i] = x[i] * ss * h->layers[l].ffn_norm[i];
        else for (int i = 0; i < D; i++) fn[i] = x[i] * ss;
        if (h->layers[l].gate && h->layers[l].up && h->layers[l].down) {
            jdo_mv(gate, h->layers[l].gate, h->layers[l].gate_dt, fn, HH, D);
            jdo_mv(up, h->layers[l].up, h->layers[l].up_dt, fn, HH, D);
            for (int i = 0; i < HH; i++) gate[i] = gate[i] / (1.0f + expf(-gate[i])) * up[i];
            jdo_mv(fo, h->layers[l].down, h->layers[l].down_dt, gate, D, HH);
            for (int i = 0; i < D; i++) x[i] += fo[i] * h->layer_focus[l];
            /* janusdoe.c:3274-3278: the learning target dy, the FFN output RMS-normalised */
            double sd = 0; for (int i = 0; i < D; i++) sd += (double)fo[i] * fo[i];
            float inv = 1.0f / (sqrtf((float)(sd / D)) + 1e-8f);
            for (int i = 0; i < D; i++) s->host_dy[i] = fo[i] * inv;
        }
        {
            int sel[JDO_MAX_EXPERTS]; float w[JDO_MAX_EXPERTS];
            int kk = jdo_host_elect(h, l, &s->consensus[l], xn, D, sel, w, trace ? &trace[l] : NULL);
            for (int ki = 0; ki < kk; ki++) {
                int e = sel[ki];
                if (!h->alive[l][e] || !h->A[l][e] || !h->B[l][e]) continue;
                const float *A = h->A[l][e], *Bm = h->B[l][e];
                float wt = h->lora_alpha * w[ki];
                memset(t, 0, (size_t)(R > 0 ? R : 1) * 4);
                for (int r = 0; r < R; r++) { float sacc = 0; for (int j = 0; j < D; j++) sacc += Bm[r * D + j] * xn[j]; t[r] = sacc; }
                for (int i = 0; i < D; i++) { float sacc = 0; for (int r = 0; r < R; r++) sacc += A[i * R + r] * t[r]; x[i] += wt * sacc; }
                s->tokens_seen[l][e]++;   /* janusdoe.c:3300 */
            }
        }
    }
    float ss = 0; for (int i = 0; i < D; i++) ss += x[i] * x[i];
    ss = 1.0f / sqrtf(ss / D + h->rms_eps);
    if (h->output_norm) for (int i = 0; i < D; i++) x[i] = x[i] * ss * h->output_norm[i];
    else for (int i = 0; i < D; i++) x[i] *= ss;
    {   /* janusdoe.c:3311-3315: the learning target x, the final hidden RMS-normalised */
        double sx = 0; for (int i = 0; i < D; i++) sx += (double)x[i] * x[i];
        float inv = 1.0f / (sqrtf((float)(sx / D)) + 1e-8f);
        for (int i = 0; i < D; i++) s->host_x[i] = x[i] * inv;
    }
    jdo_mv(logits, h->output, h->output_dt, x, h->vocab, D);
    free(x); free(t); free(xn); free(q); free(k); free(v); free(ao_in); free(ao); free(fn); free(gate); free(up); free(fo); free(att);
}

/* ============================ Hebbian --learn =========================== */
/* janusdoe.c:3091-3096 host_prophecy_debt */
static float jdo_prophecy_debt(const float *lg, int chosen, int n) {
    if (n <= 0 || chosen < 0 || chosen >= n) return 0.0f;
    float mx = lg[0]; for (int i = 1; i < n; i++) if (lg[i] > mx) mx = lg[i];
    float diff = mx - lg[chosen];
    return diff > 0.0f ? diff / (diff + 1.0f) : 0.0f;
}
#define JDO_NOTORCH_RANK 4
/* janusdoe.c:3102-3132 host_notorch_step with the global RNG and offset made explicit */
static void jdo_notorch_step(float *A, float *B, int D, int rank, const float *x, const float *dy, float signal,
                             float lr_base, uint64_t *rng, int *offset) {
    if (fabsf(signal) < 1e-8f) return;
    if (signal > 2.0f) signal = 2.0f;
    if (signal < -2.0f) signal = -2.0f;
    float lr = lr_base * signal;
    int nr = JDO_NOTORCH_RANK; if (nr > rank) nr = rank;
    int base = *offset % rank;
    float u[JDO_NOTORCH_RANK];
    for (int j = 0; j < nr; j++) {
        int r = (base + j) % rank;
        float sacc = 0; for (int i = 0; i < D; i++) sacc += B[r * D + i] * dy[i];
        sacc += jdo_rand_normal(rng) * 0.01f;
        if (sacc > 1.0f) sacc = 1.0f;
        if (sacc < -1.0f) sacc = -1.0f;
        u[j] = sacc;
    }
    for (int j = 0; j < nr; j++) {
        int r = (base + j) % rank; float ur = u[j];
        for (int i = 0; i < D; i++) { float *a = &A[i * rank + r]; *a += lr * ur * (x[i] - ur * (*a)); }
        for (int i = 0; i < D; i++) { float *b = &B[r * D + i]; *b += lr * ur * (dy[i] - ur * (*b)); }
    }
    *offset = (base + nr) % rank;
    int n = D * rank; const float cap = 0.05f;
    double sa = 0, sb = 0; for (int i = 0; i < n; i++) { sa += (double)A[i] * A[i]; sb += (double)B[i] * B[i]; }
    float ra = (float)sqrt(sa / n), rb = (float)sqrt(sb / n);
    if (ra > cap) { float f = cap / ra; for (int i = 0; i < n; i++) A[i] *= f; }
    if (rb > cap) { float f = cap / rb; for (int i = 0; i < n; i++) B[i] *= f; }
}
/* janusdoe.c:3136-3144 host_lora_poisoned */
static int jdo_lora_poisoned(const float *A, const float *B, int D, int rank) {
    int n = D * rank; double s2 = 0; float mx = 0;
    for (int i = 0; i < n; i++) { float a = A[i]; if (!isfinite(a)) return 1; float ab = fabsf(a); if (ab > mx) mx = ab; s2 += (double)a * a; }
    for (int i = 0; i < n; i++) { float b = B[i]; if (!isfinite(b)) return 1; float ab = fabsf(b); if (ab > mx) mx = ab; s2 += (double)b * b; }
    if (mx > 8.0f) return 1;
    if (sqrt(s2 / (2.0 * n)) > 5.0) return 1;
    return 0;
}
/* janusdoe.c:3420-3447 host_learn_run: fresh caches, the EMA state carried on */
int jdo_host_learn_run(jdo_host *h, jdo_host_state *s, const int *toks, int nt, float lr, uint64_t *rng,
                       int *notorch_offset) {
    size_t n = (size_t)h->n_layers * s->max_seq * h->n_kv_heads * h->head_dim;
    memset(s->kc, 0, n * 4); memset(s->vc, 0, n * 4);
    float *lg = malloc((size_t)h->vocab * 4);
    if (!lg) return 0;
    memset(s->tokens_seen, 0, sizeof(s->tokens_seen));
    int deaths = 0;
    for (int t = 0; t + 1 < nt && t < s->max_seq - 1; t++) {
        jdo_host_forward(h, s, toks[t], t, lg, NULL);
        int nxt = toks[t + 1];
        float signal = 0.0f;
        if (nxt >= 0 && nxt < h->vocab) {
            float pd = jdo_prophecy_debt(lg, nxt, h->vocab);
            signal = pd > 0.3f ? -pd : (1.0f - pd) * 0.1f;
        }
        for (int l = 0; l < h->n_layers && l < JDO_MAX_LAYERS; l++)
            for (int e = 0; e < JDO_MAX_EXPERTS; e++) {
                if (!h->alive[l][e] || s->tokens_seen[l][e] == 0 || !h->A[l][e] || !h->B[l][e]) continue;
                jdo_notorch_step(h->A[l][e], h->B[l][e], h->dim, h->lora_rank, s->host_x, s->host_dy, signal, lr,
                                 rng, notorch_offset);
                if (jdo_lora_poisoned(h->A[l][e], h->B[l][e], h->dim, h->lora_rank)) { h->alive[l][e] = 0; deaths++; }
                s->tokens_seen[l][e] = 0;
            }
    }
    free(lg);
    return deaths;
}

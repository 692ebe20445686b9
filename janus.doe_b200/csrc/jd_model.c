/*
 * jd_model.c — host-side model code of the B200 engine: the reference's model structs,
 * synthetic weights, and both GGUF formats (own-model export/load and the host-model
 * mmap loader), plus the synthetic quantised-GGUF generator used by the benchmarks.
 * No CUDA here; jdg_engine.cu uploads what these functions build.
 */
#define _GNU_SOURCE
#include "../../include/jdgpu.h"
#include "jd_quant.h"
#include <fcntl.h>
#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

/* ================================ RNG =================================== */
/* splitmix64 seed mixer (Steele, Lea & Flood 2014); xorshift64 state 0 is a fixed point */
static uint64_t jd_splitmix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    z = z ^ (z >> 31);
    return z ? z : 1;
}
/* janusdoe.c:191-193: xorshift64 (13, 7, 17), 31-bit uniform, Box-Muller cosine branch */
static uint64_t jd_xs(uint64_t *s) { uint64_t x = *s; x ^= x << 13; x ^= x >> 7; x ^= x << 17; *s = x; return x; }
static float jd_uni(uint64_t *s) { return (float)(jd_xs(s) & 0x7FFFFFFF) / (float)0x7FFFFFFF; }
static float jd_normal(uint64_t *s) {
    float u1 = jd_uni(s), u2 = jd_uni(s);
    if (u1 < 1e-10f) u1 = 1e-10f;
    return sqrtf(-2.0f * logf(u1)) * cosf(6.2831853f * u2);
}

/* ============================== own model =============================== */
int jd_config_from_depth(int depth, jd_config *c) {
    if (!c || depth < 1 || depth > JD_MAX_LAYERS) return JD_EINVAL;
    memset(c, 0, sizeof(*c));
    c->depth = depth;
    c->dim = ((depth * 64 + 63) / 64) * 64;
    if (c->dim < 128) c->dim = 128;
    if (c->dim > 768) c->dim = 768;
    c->head_dim = 64;
    c->n_heads = c->dim / c->head_dim;
    if (c->n_heads < 1) c->n_heads = 1;
    if (c->dim <= 384) c->n_kv_heads = c->n_heads;
    else {
        c->n_kv_heads = c->n_heads / 2;
        if (c->n_kv_heads < 1) c->n_kv_heads = 1;
        while (c->n_heads % c->n_kv_heads != 0 && c->n_kv_heads > 1) c->n_kv_heads--;
    }
    c->initial_experts = (depth <= 4) ? 4 : (depth <= 8) ? 6 : 8;
    c->hidden_dim = (int)(c->dim * 1.5f);
    c->hidden_dim = ((c->hidden_dim + 63) / 64) * 64;
    c->seq_len = 256;
    c->norm_eps = 1e-5f;
    c->rope_theta = 10000.0f;
    c->attn_clamp = 30.0f;
    c->active_depth = depth;
    c->vocab_size = 258 + (depth <= 4 ? 2000 : depth <= 8 ? 4000 : 8000);
    return JD_OK;
}

static int jd_cfg_ok(const jd_config *c) {
    return c->depth >= 1 && c->depth <= JD_MAX_LAYERS && c->dim > 0 && c->head_dim > 0 && c->n_heads > 0 &&
           c->n_kv_heads > 0 && c->n_heads % c->n_kv_heads == 0 && c->hidden_dim > 0 && c->vocab_size > 0 &&
           c->seq_len > 0 && c->initial_experts >= 0 && c->initial_experts <= JD_MAX_EXPERTS && c->head_dim % 2 == 0;
}

static int jd_alloc_expert(jd_layer *L, int e, int D, int H) {
    L->w_gate[e] = calloc((size_t)H * D, 4);
    L->w_up[e] = calloc((size_t)H * D, 4);
    L->w_down[e] = calloc((size_t)D * H, 4);
    if (!L->w_gate[e] || !L->w_up[e] || !L->w_down[e]) return JD_ENOMEM;
    L->alive[e] = 1;
    return JD_OK;
}
static void jd_kill_expert(jd_layer *L, int e) {
    free(L->w_gate[e]); free(L->w_up[e]); free(L->w_down[e]);
    L->w_gate[e] = L->w_up[e] = L->w_down[e] = NULL;
    L->alive[e] = 0;
}

int jd_model_alloc(jd_model *m, const jd_config *c) {
    if (!m || !c || !jd_cfg_ok(c)) return JD_EINVAL;
    memset(m, 0, sizeof(*m));
    m->c = *c;
    int D = c->dim, qd = c->n_heads * c->head_dim, kd = c->n_kv_heads * c->head_dim, H = c->hidden_dim;
    size_t V = (size_t)c->vocab_size;
    m->tok_emb = calloc(V * D, 4);
    m->output = calloc(V * D, 4);
    m->output_norm = malloc((size_t)D * 4);
    if (!m->tok_emb || !m->output || !m->output_norm) goto oom;
    for (int i = 0; i < D; i++) m->output_norm[i] = 1.0f;
    for (int l = 0; l < c->depth; l++) {
        jd_layer *L = &m->layers[l];
        L->attn_norm = malloc((size_t)D * 4);
        L->ffn_norm = malloc((size_t)D * 4);
        L->wq = calloc((size_t)qd * D, 4);
        L->wk = calloc((size_t)kd * D, 4);
        L->wv = calloc((size_t)kd * D, 4);
        L->wo = calloc((size_t)D * qd, 4);
        L->w_vote = calloc((size_t)JD_MAX_EXPERTS * D, 4);
        if (!L->attn_norm || !L->ffn_norm || !L->wq || !L->wk || !L->wv || !L->wo || !L->w_vote) goto oom;
        for (int i = 0; i < D; i++) L->attn_norm[i] = L->ffn_norm[i] = 1.0f;
        L->consensus = 0.5f;
        L->temperature = 0.0f;
        for (int e = 0; e < c->initial_experts; e++)
            if (jd_alloc_expert(L, e, D, H) != JD_OK) goto oom;
    }
    return JD_OK;
oom:
    jd_model_free(m);
    return JD_ENOMEM;
}

void jd_model_free(jd_model *m) {
    if (!m) return;
    free(m->tok_emb); free(m->output); free(m->output_norm);
    for (int l = 0; l < JD_MAX_LAYERS; l++) {
        jd_layer *L = &m->layers[l];
        free(L->attn_norm); free(L->ffn_norm); free(L->wq); free(L->wk); free(L->wv); free(L->wo); free(L->w_vote);
        for (int e = 0; e < JD_MAX_EXPERTS; e++) jd_kill_expert(L, e);
    }
    memset(m, 0, sizeof(*m));
}

static void jd_fill(float *p, size_t n, uint64_t *s, float std) { for (size_t i = 0; i < n; i++) p[i] = jd_normal(s) * std; }

int jd_model_fill_seeded(jd_model *m, uint64_t seed, float std, int draw_masks) {
    if (!m || !m->tok_emb) return JD_EINVAL;
    const jd_config *c = &m->c;
    int D = c->dim, qd = c->n_heads * c->head_dim, kd = c->n_kv_heads * c->head_dim, H = c->hidden_dim;
    size_t V = (size_t)c->vocab_size;
    uint64_t s = jd_splitmix64(seed);
    jd_fill(m->tok_emb, V * D, &s, std);
    jd_fill(m->output, V * D, &s, std);
    for (int l = 0; l < c->depth; l++) {
        jd_layer *L = &m->layers[l];
        jd_fill(L->wq, (size_t)qd * D, &s, std);
        jd_fill(L->wk, (size_t)kd * D, &s, std);
        jd_fill(L->wv, (size_t)kd * D, &s, std);
        jd_fill(L->wo, (size_t)D * qd, &s, std);
        jd_fill(L->w_vote, (size_t)JD_MAX_EXPERTS * D, &s, std);
        for (int e = 0; e < c->initial_experts; e++) {
            if (!L->alive[e]) return JD_ESTATE;
            jd_fill(L->w_gate[e], (size_t)H * D, &s, std);
            jd_fill(L->w_up[e], (size_t)H * D, &s, std);
            jd_fill(L->w_down[e], (size_t)D * H, &s, std);
        }
    }
    if (draw_masks) {
        int n0 = c->initial_experts, lo = n0 - 3 < 2 ? 2 : n0 - 3;
        if (n0 < 2) return JD_EINVAL;
        for (int l = 0; l < c->depth; l++) {
            jd_layer *L = &m->layers[l];
            int target = lo + (int)(jd_xs(&s) % (uint64_t)(n0 - lo + 1)), n = n0;
            while (n > target) {
                int e = (int)(jd_xs(&s) % (uint64_t)n0);
                if (L->alive[e]) { jd_kill_expert(L, e); n--; }
            }
        }
    }
    return JD_OK;
}

/* ---- GGUF writing helpers ---- */
static int w32(FILE *f, uint32_t v) { return fwrite(&v, 4, 1, f) == 1; }
static int w64(FILE *f, uint64_t v) { return fwrite(&v, 8, 1, f) == 1; }
static int wstr(FILE *f, const char *s) { uint64_t l = strlen(s); return w64(f, l) && fwrite(s, 1, l, f) == l; }
static int wkv_s(FILE *f, const char *k, const char *v) { return wstr(f, k) && w32(f, 8) && wstr(f, v); }
static int wkv_u(FILE *f, const char *k, uint32_t v) { return wstr(f, k) && w32(f, 4) && w32(f, v); }
static int wkv_f(FILE *f, const char *k, float v) { return wstr(f, k) && w32(f, 6) && fwrite(&v, 4, 1, f) == 1; }

typedef struct { const char *name; const float *data; uint64_t rows, cols; } jd_own_t;

/* Tensor list in export order (janusdoe.c:1797-1812): shapes as the reference's Tensor rows/cols. */
static int jd_own_tensors(const jd_model *m, jd_own_t *t, char (*names)[96]) {
    const jd_config *c = &m->c;
    int D = c->dim, qd = c->n_heads * c->head_dim, kd = c->n_kv_heads * c->head_dim, H = c->hidden_dim, n = 0;
#define ADD(nm, p, r, cc) do { snprintf(names[n], 96, "%s", nm); t[n].name = names[n]; t[n].data = (p); t[n].rows = (r); t[n].cols = (cc); n++; } while (0)
    ADD("token_embd.weight", m->tok_emb, c->vocab_size, D);
    ADD("output_norm.weight", m->output_norm, 1, D);
    ADD("output.weight", m->output, c->vocab_size, D);
    char nm[96];
    for (int l = 0; l < c->depth; l++) {
        const jd_layer *L = &m->layers[l];
        snprintf(nm, 96, "blk.%d.attn_norm.weight", l); ADD(nm, L->attn_norm, 1, D);
        snprintf(nm, 96, "blk.%d.attn_q.weight", l); ADD(nm, L->wq, qd, D);
        snprintf(nm, 96, "blk.%d.attn_k.weight", l); ADD(nm, L->wk, kd, D);
        snprintf(nm, 96, "blk.%d.attn_v.weight", l); ADD(nm, L->wv, kd, D);
        snprintf(nm, 96, "blk.%d.attn_output.weight", l); ADD(nm, L->wo, D, qd);
        snprintf(nm, 96, "blk.%d.ffn_norm.weight", l); ADD(nm, L->ffn_norm, 1, D);
        snprintf(nm, 96, "blk.%d.ffn_gate_inp.weight", l); ADD(nm, L->w_vote, JD_MAX_EXPERTS, D);
        for (int e = 0; e < JD_MAX_EXPERTS; e++) {
            if (!L->alive[e]) continue;
            snprintf(nm, 96, "blk.%d.ffn_gate.%d.weight", l, e); ADD(nm, L->w_gate[e], H, D);
            snprintf(nm, 96, "blk.%d.ffn_up.%d.weight", l, e); ADD(nm, L->w_up[e], H, D);
            snprintf(nm, 96, "blk.%d.ffn_down.%d.weight", l, e); ADD(nm, L->w_down[e], D, H);
        }
    }
#undef ADD
    return n;
}

int jd_model_export_gguf(const jd_model *m, const char *path) {
    if (!m || !path || !m->tok_emb) return JD_EINVAL;
    const jd_config *c = &m->c;
    int maxn = 3 + c->depth * (7 + 3 * JD_MAX_EXPERTS);
    jd_own_t *t = calloc(maxn, sizeof(*t));
    char (*names)[96] = calloc(maxn, 96);
    if (!t || !names) { free(t); free(names); return JD_ENOMEM; }
    int nt = jd_own_tensors(m, t, names);
    FILE *f = fopen(path, "wb");
    if (!f) { free(t); free(names); return JD_EIO; }
    int ok = w32(f, 0x46554747) && w32(f, 3) && w64(f, (uint64_t)nt) && w64(f, 13);
    ok = ok && wkv_s(f, "general.architecture", "llama") && wkv_s(f, "general.name", "m");
    ok = ok && wkv_u(f, "llama.block_count", c->depth) && wkv_u(f, "llama.embedding_length", c->dim);
    ok = ok && wkv_u(f, "llama.attention.head_count", c->n_heads) && wkv_u(f, "llama.attention.head_count_kv", c->n_kv_heads);
    ok = ok && wkv_u(f, "llama.feed_forward_length", c->hidden_dim) && wkv_u(f, "llama.context_length", c->seq_len);
    ok = ok && wkv_f(f, "llama.attention.layer_norm_rms_epsilon", c->norm_eps) && wkv_f(f, "llama.rope.freq_base", c->rope_theta);
    ok = ok && wkv_u(f, "m.max_experts", JD_MAX_EXPERTS) && wkv_u(f, "m.initial_experts", c->initial_experts);
    ok = ok && wkv_s(f, "tokenizer.ggml.model", "gpt2");
    uint64_t off = 0;
    for (int i = 0; i < nt && ok; i++) {
        ok = wstr(f, t[i].name);
        if (t[i].rows > 1) ok = ok && w32(f, 2) && w64(f, t[i].cols) && w64(f, t[i].rows);
        else ok = ok && w32(f, 1) && w64(f, t[i].cols);
        ok = ok && w32(f, 0) && w64(f, off);
        off += t[i].rows * t[i].cols * 4;
    }
    long p = ftell(f), al = ((p + 31) / 32) * 32;
    for (long i = p; i < al && ok; i++) ok = fputc(0, f) != EOF;
    for (int i = 0; i < nt && ok; i++) ok = fwrite(t[i].data, 4, t[i].rows * t[i].cols, f) == t[i].rows * t[i].cols;
    if (fclose(f) != 0) ok = 0;
    free(t); free(names);
    return ok ? JD_OK : JD_EIO;
}

int jd_model_load_gguf(jd_model *m, const char *path) {
    if (!m || !path || !m->tok_emb) return JD_EINVAL;
    jd_config *c = &m->c;
    FILE *f = fopen(path, "rb");
    if (!f) return JD_EIO;
    int rc = JD_EFORMAT;
    struct { char name[96]; uint64_t nbytes, off; } *ti = NULL;
    uint32_t magic = 0, ver = 0;
    uint64_t n_tensors = 0, n_kv = 0;
    if (fread(&magic, 4, 1, f) != 1 || magic != 0x46554747) goto done;
    if (fread(&ver, 4, 1, f) != 1 || fread(&n_tensors, 8, 1, f) != 1 || fread(&n_kv, 8, 1, f) != 1) goto done;
    int is_ours = 0, fdepth = 0, fdim = 0;
    for (uint64_t i = 0; i < n_kv; i++) {
        uint64_t kl; char key[256] = {0}; uint32_t vt;
        if (fread(&kl, 8, 1, f) != 1 || kl > 255 || fread(key, 1, kl, f) != kl || fread(&vt, 4, 1, f) != 1) goto done;
        if (vt == 8) {
            uint64_t vl; char val[256] = {0};
            if (fread(&vl, 8, 1, f) != 1) goto done;
            size_t rl = vl > 255 ? 255 : (size_t)vl;
            if (fread(val, 1, rl, f) != rl) goto done;
            if (vl > 255 && fseek(f, (long)(vl - 255), SEEK_CUR) != 0) goto done;
            if (strstr(key, "general.name") && strcmp(val, "m") == 0) is_ours = 1;
        } else if (vt == 4) {
            uint32_t v; if (fread(&v, 4, 1, f) != 1) goto done;
            if (strstr(key, "block_count")) fdepth = (int)v;
            if (strstr(key, "embedding_length")) fdim = (int)v;
        } else if (vt == 6) {
            float v; if (fread(&v, 4, 1, f) != 1) goto done;
        } else goto done;
    }
    if (!is_ours || fdepth != c->depth || fdim != c->dim) { rc = JD_EFORMAT; goto done; }
    if (n_tensors > 100000) goto done;
    ti = calloc(n_tensors ? n_tensors : 1, sizeof(*ti));
    if (!ti) { rc = JD_ENOMEM; goto done; }
    for (uint64_t i = 0; i < n_tensors; i++) {
        uint64_t nl, sz = 1; uint32_t nd, dt;
        if (fread(&nl, 8, 1, f) != 1 || nl > 95 || fread(ti[i].name, 1, nl, f) != nl) goto done;
        ti[i].name[nl] = 0;
        if (fread(&nd, 4, 1, f) != 1 || nd > 4) goto done;
        for (uint32_t d = 0; d < nd; d++) { uint64_t dv; if (fread(&dv, 8, 1, f) != 1) goto done; sz *= dv; }
        if (fread(&dt, 4, 1, f) != 1 || fread(&ti[i].off, 8, 1, f) != 1) goto done;
        ti[i].nbytes = sz * 4;
    }
    long hdr = ftell(f), data_start = ((hdr + 31) / 32) * 32;
    if (fseek(f, 0, SEEK_END) != 0) goto done;
    long fsz = ftell(f);
    if (data_start > fsz) goto done;
    uint64_t region = (uint64_t)(fsz - data_start);
    int have_emb = 0;
    for (uint64_t i = 0; i < n_tensors; i++) {
        if (ti[i].off > region || ti[i].nbytes > region - ti[i].off) goto done;
        if (strcmp(ti[i].name, "token_embd.weight") == 0) {
            have_emb = 1;
            if (ti[i].nbytes != (uint64_t)c->vocab_size * c->dim * 4) goto done;
        }
    }
    if (!have_emb) goto done;
    int loaded = 0, tok_ok = 0;
    int D = c->dim, qd = c->n_heads * c->head_dim, kd = c->n_kv_heads * c->head_dim, H = c->hidden_dim;
#define FIND(nm) ({ long _k = -1; for (uint64_t _i = 0; _i < n_tensors; _i++) if (!strcmp(ti[_i].name, (nm))) { _k = (long)_i; break; } _k; })
#define LOADP(ptr, nelem, nm) ({ int _ok = 0; long _k = FIND(nm); \
        if (_k >= 0 && (ptr) && ti[_k].nbytes == (uint64_t)(nelem) * 4 && fseek(f, data_start + (long)ti[_k].off, SEEK_SET) == 0 && \
            fread((ptr), 4, (nelem), f) == (size_t)(nelem)) { loaded++; _ok = 1; } _ok; })
    tok_ok = LOADP(m->tok_emb, (size_t)c->vocab_size * D, "token_embd.weight");
    LOADP(m->output_norm, (size_t)D, "output_norm.weight");
    LOADP(m->output, (size_t)c->vocab_size * D, "output.weight");
    char n[96];
    for (int l = 0; l < c->depth; l++) {
        jd_layer *L = &m->layers[l];
        snprintf(n, 96, "blk.%d.attn_norm.weight", l); LOADP(L->attn_norm, (size_t)D, n);
        snprintf(n, 96, "blk.%d.attn_q.weight", l); LOADP(L->wq, (size_t)qd * D, n);
        snprintf(n, 96, "blk.%d.attn_k.weight", l); LOADP(L->wk, (size_t)kd * D, n);
        snprintf(n, 96, "blk.%d.attn_v.weight", l); LOADP(L->wv, (size_t)kd * D, n);
        snprintf(n, 96, "blk.%d.attn_output.weight", l); LOADP(L->wo, (size_t)D * qd, n);
        snprintf(n, 96, "blk.%d.ffn_norm.weight", l); LOADP(L->ffn_norm, (size_t)D, n);
        snprintf(n, 96, "blk.%d.ffn_gate_inp.weight", l); LOADP(L->w_vote, (size_t)JD_MAX_EXPERTS * D, n);
        int snap[JD_MAX_EXPERTS] = {0};
        for (int e = 0; e < JD_MAX_EXPERTS; e++) {
            char ng[96], nu[96], nd[96];
            snprintf(ng, 96, "blk.%d.ffn_gate.%d.weight", l, e);
            snprintf(nu, 96, "blk.%d.ffn_up.%d.weight", l, e);
            snprintf(nd, 96, "blk.%d.ffn_down.%d.weight", l, e);
            if (FIND(ng) < 0 || FIND(nu) < 0 || FIND(nd) < 0) continue;
            if (!L->alive[e] && jd_alloc_expert(L, e, D, H) != JD_OK) { rc = JD_ENOMEM; goto done; }
            int ok = LOADP(L->w_gate[e], (size_t)H * D, ng) + LOADP(L->w_up[e], (size_t)H * D, nu) + LOADP(L->w_down[e], (size_t)D * H, nd);
            if (ok == 3) snap[e] = 1; else jd_kill_expert(L, e);
        }
        for (int e = 0; e < JD_MAX_EXPERTS; e++) if (L->alive[e] && !snap[e]) jd_kill_expert(L, e);
    }
#undef LOADP
#undef FIND
    rc = (tok_ok && loaded >= 2 + 6 * c->depth) ? JD_OK : JD_EFORMAT;
done:
    free(ti);
    fclose(f);
    return rc;
}

/* ============================= packed formats =========================== */
/* Block layouts, field extraction and the whole-tensor decoder: jd_quant.h */
/* float -> half, round to nearest even (IEEE 754 binary16) */
static uint16_t jd_f2h(float v) {
    uint32_t x; memcpy(&x, &v, 4);
    uint32_t sign = (x >> 16) & 0x8000, e8 = (x >> 23) & 0xFF, mant = x & 0x7FFFFF;
    if (e8 == 0xFF) return (uint16_t)(sign | 0x7C00 | (mant ? 0x200 : 0));
    int e = (int)e8 - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000;
        int shift = 14 - e;
        uint32_t h = mant >> shift, rem = mant & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (mant >> 13), rem = mant & 0x1FFF;
    if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;
    return (uint16_t)(sign | h);
}
/* janusdoe.c:2674-2680 jd_pq_for: dtypes with a row kernel (here: a GPU kernel) */
static int jd_has_rows(int dt, int c) {
    return ((dt == JD_Q8_0 || dt == JD_Q4_0 || dt == JD_Q5_0) && c % 32 == 0) ||
           ((dt == JD_Q4_K || dt == JD_Q6_K) && c % 256 == 0) || (dt == JD_F16 && c % 4 == 0);
}
int jd_dequant(const void *src, float *out, uint64_t n, int dt) {
    if (!src || !out) return JD_EINVAL;
    return jdq_decode((const uint8_t *)src, out, n, dt) == 0 ? JD_OK : JD_EUNSUPPORTED;
}

int jd_tp_shard_of(const jd_host_model *h, int rank, int world, jd_tp_shard *out) {
    if (!h || !out || world < 1 || rank < 0 || rank >= world || h->n_heads < 1 || h->n_kv_heads < 1) return JD_EINVAL;
    if (h->n_heads % world || h->n_kv_heads % world || h->hidden % world) return JD_EINVAL;
    out->q_heads = h->n_heads / world;
    out->q_head0 = rank * out->q_heads;
    out->kv_heads = h->n_kv_heads / world;
    out->kv_head0 = rank * out->kv_heads;
    out->hidden = h->hidden / world;
    out->hidden0 = rank * out->hidden;
    const int per = (h->vocab + world - 1) / world;   /* ceil: the last rank may hold fewer */
    out->vocab0 = rank * per;
    out->vocab = out->vocab0 >= h->vocab ? 0 : (out->vocab0 + per > h->vocab ? h->vocab - out->vocab0 : per);
    return JD_OK;
}

/* ============================== host model ============================== */
typedef struct {
    uint8_t *map; size_t map_size;   /* file mapping, or NULL */
    void **owned; int n_owned, cap_owned;
    int *vocab_slot;                 /* open-addressing index of the token strings (-1 empty) */
    uint32_t vocab_mask;
} jd_host_priv;

static int jd_priv_own(jd_host_priv *p, void *buf) {
    if (p->n_owned == p->cap_owned) {
        int nc = p->cap_owned ? p->cap_owned * 2 : 64;
        void **o = realloc(p->owned, (size_t)nc * sizeof(void *));
        if (!o) return JD_ENOMEM;
        p->owned = o; p->cap_owned = nc;
    }
    p->owned[p->n_owned++] = buf;
    return JD_OK;
}

static int jd_rope_norm_for_arch(const char *arch) {
    return !strcmp(arch, "llama") || !strcmp(arch, "mistral") || !strcmp(arch, "mistral3") || !strcmp(arch, "mistral4");
}

/* janusdoe.c:2817-2833 jd_host_resolve */
static const void *jd_resolve(jd_host_priv *pv, const uint8_t *raw, const uint8_t *pend, int dt, uint64_t ne, int c,
                              int want_f32, int *out_dt) {
    *out_dt = 0;
    uint64_t bytes = jdq_bytes(dt, ne);
    if (dt != 0 && bytes == 0) return NULL;
    if (bytes == 0) bytes = ne * 4;
    if (raw > pend || bytes > (uint64_t)(pend - raw)) return NULL;
    if (dt == 0) return raw;
    if (!want_f32 && jd_has_rows(dt, c)) { *out_dt = dt; return raw; }
    float *buf = malloc(ne * 4);
    if (!buf) return NULL;
    if (jdq_decode(raw, buf, ne, dt) != 0 || jd_priv_own(pv, buf) != JD_OK) { free(buf); return NULL; }
    return buf;
}

static int jd_host_lora_alloc(jd_host_model *h, int n_alive) {
    jd_host_priv *pv = (jd_host_priv *)h->priv;
    int D = h->dim, R = h->lora_rank;
    for (int l = 0; l < h->n_layers && l < JD_MAX_LAYERS; l++) {
        if (!h->w_vote[l]) {
            h->w_vote[l] = calloc((size_t)JD_MAX_EXPERTS * D, 4);
            if (!h->w_vote[l] || jd_priv_own(pv, h->w_vote[l]) != JD_OK) return JD_ENOMEM;
        }
        for (int e = 0; e < JD_MAX_EXPERTS; e++) {
            if (e < n_alive && !h->A[l][e]) {
                h->A[l][e] = calloc((size_t)D * R, 4);
                h->B[l][e] = calloc((size_t)R * D, 4);
                if (!h->A[l][e] || !h->B[l][e]) return JD_ENOMEM;
                if (jd_priv_own(pv, h->A[l][e]) != JD_OK || jd_priv_own(pv, h->B[l][e]) != JD_OK) return JD_ENOMEM;
            }
            h->alive[l][e] = e < n_alive && h->A[l][e] != NULL;
        }
        h->consensus0[l] = 0.5f; h->attention_bias[l] = 0.0f; h->layer_focus[l] = 1.0f;
    }
    return JD_OK;
}

/* Finish a parsed host: tied output, essentials, standard FFN, RoPE pairing, LoRA slots
 * (janusdoe.c:2985-3029). */
static int jd_host_finish(jd_host_model *h, int rope_override, int lora_rank) {
    if (!h->output && h->tok_emb) { h->output = h->tok_emb; h->output_dt = 0; }
    if (!h->tok_emb || !h->output || !h->output_norm) return JD_EFORMAT;
    int has_ffn = 0;
    for (int l = 0; l < h->n_layers && l < JD_MAX_LAYERS; l++)
        if (h->layers[l].gate && h->layers[l].up && h->layers[l].down) has_ffn = 1;
    if (!has_ffn) return JD_EFORMAT;
    h->rope_norm = rope_override >= 0 ? rope_override : jd_rope_norm_for_arch(h->arch);
    h->lora_rank = lora_rank;
    h->lora_alpha = 0.1f;
    return jd_host_lora_alloc(h, 4);
}

/* ---------------------------------------------------------------------------------
 * Host tokenizer (janusdoe.c:3329-3356): whole-word lookups of the GGUF vocabulary.
 * The vocabulary is indexed once at load in an open-addressing hash table (FNV-1a over
 * the token's bytes up to its first NUL, as the loader stores it); every token string maps
 * to its lowest id, which is what a first-match scan over the ids returns. */
#define JD_GSPACE "\xc4\xa0" /* "Ġ", the byte-level BPE space marker (UTF-8 C4 A0) */
static uint64_t jd_fnv(uint64_t h, const unsigned char *p, size_t n) {
    for (size_t i = 0; i < n; i++) h = (h ^ p[i]) * 0x100000001b3ull;
    return h;
}
static const uint64_t JD_FNV0 = 0xcbf29ce484222325ull;

/* Token text == (space marker if sp) + w[0..n), compared without building the key. */
static int jd_tok_eq(const char *tok, int sp, const char *w, size_t n) {
    if (sp) {
        if ((unsigned char)tok[0] != 0xC4 || (unsigned char)tok[1] != 0xA0) return 0;
        tok += 2;
    }
    return strncmp(tok, w, n) == 0 && tok[n] == '\0';
}

static int jd_vocab_index_build(jd_host_model *h) {
    jd_host_priv *pv = (jd_host_priv *)h->priv;
    if (!pv || !h->vocab_tokens || h->n_vocab_tokens <= 0) return JD_OK;
    uint32_t cap = 64;
    while (cap < 2u * (uint32_t)h->n_vocab_tokens) cap <<= 1;
    pv->vocab_slot = malloc((size_t)cap * sizeof(int));
    if (!pv->vocab_slot) return JD_ENOMEM;
    for (uint32_t i = 0; i < cap; i++) pv->vocab_slot[i] = -1;
    pv->vocab_mask = cap - 1;
    for (int id = 0; id < h->n_vocab_tokens; id++) {
        const char *t = h->vocab_tokens[id];
        if (!t) continue;
        size_t n = strlen(t);
        uint32_t i = (uint32_t)jd_fnv(JD_FNV0, (const unsigned char *)t, n) & pv->vocab_mask;
        for (;; i = (i + 1) & pv->vocab_mask) {
            int o = pv->vocab_slot[i];
            if (o < 0) { pv->vocab_slot[i] = id; break; }
            if (strcmp(h->vocab_tokens[o], t) == 0) break; /* a lower id already holds it */
        }
    }
    return JD_OK;
}

/* Lowest id whose text is (space marker if sp) + w[0..n), or -1. */
static int jd_vocab_find(const jd_host_model *h, int sp, const char *w, size_t n) {
    const jd_host_priv *pv = (const jd_host_priv *)h->priv;
    if (!pv || !pv->vocab_slot) return -1;
    uint64_t hv = sp ? jd_fnv(JD_FNV0, (const unsigned char *)JD_GSPACE, 2) : JD_FNV0;
    hv = jd_fnv(hv, (const unsigned char *)w, n);
    for (uint32_t i = (uint32_t)hv & pv->vocab_mask;; i = (i + 1) & pv->vocab_mask) {
        int o = pv->vocab_slot[i];
        if (o < 0) return -1;
        if (jd_tok_eq(h->vocab_tokens[o], sp, w, n)) return o;
    }
}

int jd_host_tokenize(const jd_host_model *h, const char *text, int *out, int max) {
    if (!h || !text || !out || max < 0) return JD_EINVAL;
    int n = 0;
    const char *w = text;
    while (n < max) {
        while (*w == ' ') w++;
        if (!*w) break;
        const char *end = w;
        while (*end && *end != ' ') end++;
        const size_t len = (size_t)(end - w), key = len > 120 ? 120 : len; /* words look up by <= 120 bytes */
        int id = jd_vocab_find(h, 1, w, key);                              /* "Ġword" */
        if (id < 0) id = jd_vocab_find(h, 0, w, key);                      /* "word" */
        if (id >= 0) out[n++] = id;
        else /* byte by byte, the whole word, bytes without a token skipped */
            for (const char *c = w; c < end && n < max; c++) {
                const int ci = jd_vocab_find(h, 0, c, 1);
                if (ci >= 0) out[n++] = ci;
            }
        w = end;
    }
    return n;
}

int jd_host_token_text(const jd_host_model *h, int id, char *buf, int cap) {
    if (!h || !buf || cap < 1) return JD_EINVAL;
    int n = 0;
    if (id < 0 || id >= h->n_vocab_tokens || !h->vocab_tokens || !h->vocab_tokens[id]) {
        n = snprintf(buf, (size_t)cap, "<%d>", id);
        return n < cap ? n : cap - 1;
    }
    const unsigned char *s = (const unsigned char *)h->vocab_tokens[id];
    for (int i = 0; s[i] && n < cap - 1; i++) {
        if (s[i] == 0xC4 && (s[i + 1] == 0xA0 || s[i + 1] == 0x8A)) { /* Ġ space, Ċ newline */
            buf[n++] = s[i + 1] == 0xA0 ? ' ' : '\n';
            i++;
        } else if (s[i] >= 32 && s[i] < 127) {
            buf[n++] = (char)s[i];
        }
    }
    buf[n] = '\0';
    return n;
}

int jd_host_load_gguf(jd_host_model *h, const char *path, int rope_override, int lora_rank) {
    if (!h || !path || lora_rank < 1 || lora_rank > 256) return JD_EINVAL;
    memset(h, 0, sizeof(*h));
    h->bos = h->eos = -1;
    jd_host_priv *pv = calloc(1, sizeof(*pv));
    if (!pv) return JD_ENOMEM;
    h->priv = pv;
    int fd = open(path, O_RDONLY);
    if (fd < 0) { jd_host_free(h); return JD_EIO; }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) { close(fd); jd_host_free(h); return st.st_size < 24 ? JD_EFORMAT : JD_EIO; }
    pv->map_size = (size_t)st.st_size;
    void *mp = mmap(NULL, pv->map_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (mp == MAP_FAILED) { jd_host_free(h); return JD_EIO; }
    pv->map = (uint8_t *)mp;
    const uint8_t *p = pv->map, *pend = pv->map + pv->map_size;
    int rc = JD_EFORMAT;
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
        if (klen > 255) key[0] = 0; else { memcpy(key, p, klen); key[klen] = 0; }
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
                int is_tok = strstr(key, "tokenizer.ggml.tokens") != NULL && alen > 0 && alen < 1000000 && !h->vocab_tokens;
                if (is_tok) { h->vocab_tokens = calloc(alen, sizeof(char *)); if (h->vocab_tokens) h->n_vocab_tokens = (int)alen; }
                for (uint64_t a = 0; a < alen; a++) {
                    RD(uint64_t, sl);
                    if (sl > 1000000) goto bail;
                    NEED(sl);
                    if (is_tok && h->vocab_tokens) {
                        char *s = malloc(sl + 1);
                        if (s) { memcpy(s, p, sl); s[sl] = 0; }
                        h->vocab_tokens[a] = s;
                    }
                    p += sl;
                }
            } else {
                uint64_t esz = (at == 0 || at == 1 || at == 7) ? 1 : (at == 2 || at == 3) ? 2 : (at == 4 || at == 5 || at == 6) ? 4 : (at == 10 || at == 11 || at == 12) ? 8 : 0;
                if (esz == 0 || alen > ((uint64_t)1 << 40)) goto bail;
                NEED(alen * esz); p += alen * esz;
            }
        } else { NEED(4); p += 4; }
    }
    if (h->dim == 0 || h->dim > 16384 || h->n_layers == 0) goto bail;
    if (h->n_heads == 0) h->n_heads = h->dim / 64;
    if (h->n_heads == 0) goto bail;
    if (h->n_kv_heads == 0) h->n_kv_heads = h->n_heads;
    if (h->head_dim == 0) h->head_dim = h->dim / h->n_heads;
    if (h->hidden == 0) h->hidden = h->dim * 4;
    if (h->rope_theta == 0.0f) h->rope_theta = 10000.0f;
    if (h->rms_eps == 0.0f) h->rms_eps = 1e-6f;
    if (n_tensors > 10000) goto bail;
    ti = calloc(n_tensors ? n_tensors : 1, sizeof(*ti));
    if (!ti) { rc = JD_ENOMEM; goto bail; }
    for (uint64_t i = 0; i < n_tensors; i++) {
        RD(uint64_t, nlen);
        if (nlen > 256) goto bail;
        int nl = nlen < 95 ? (int)nlen : 95;
        NEED(nlen); memcpy(ti[i].name, p, nl); ti[i].name[nl] = 0; p += nlen;
        { RD(uint32_t, nd); ti[i].ndim = nd; }
        if (ti[i].ndim > 4) goto bail;
        for (uint32_t d = 0; d < ti[i].ndim; d++) { RD(uint64_t, dv); ti[i].dims[d] = dv; }
        { RD(uint32_t, dt); ti[i].dtype = dt; }
        { RD(uint64_t, of); ti[i].off = of; }
    }
    {
        uint64_t hdr = (uint64_t)(p - pv->map), data_start = ((hdr + 31) / 32) * 32;
        for (uint64_t i = 0; i < n_tensors; i++) {
            int dt = (int)ti[i].dtype, wdt = 0;
            if (data_start > pv->map_size || ti[i].off > pv->map_size - data_start) continue;
            const uint8_t *raw = pv->map + data_start + ti[i].off;
            uint64_t ne = 1;
            for (uint32_t d = 0; d < ti[i].ndim; d++) ne *= ti[i].dims[d];
            int c = ti[i].ndim > 0 ? (int)ti[i].dims[0] : 0;
            const char *n = ti[i].name;
            if (!strcmp(n, "token_embd.weight")) {
                h->tok_emb = jd_resolve(pv, raw, pend, dt, ne, c, 1, &wdt);
                if (h->vocab == 0) h->vocab = (int)ti[i].dims[1];
            } else if (!strcmp(n, "output_norm.weight")) h->output_norm = jd_resolve(pv, raw, pend, dt, ne, c, 1, &wdt);
            else if (!strcmp(n, "output.weight")) h->output = jd_resolve(pv, raw, pend, dt, ne, c, 0, &h->output_dt);
            else {
                int l = -1;
                sscanf(n, "blk.%d.", &l);
                if (l >= 0 && l < JD_MAX_LAYERS && l < h->n_layers) {
                    jd_host_layer *L = &h->layers[l];
                    if (strstr(n, "attn_q.weight")) L->wq = jd_resolve(pv, raw, pend, dt, ne, c, 0, &L->wq_dt);
                    else if (strstr(n, "attn_k.weight")) L->wk = jd_resolve(pv, raw, pend, dt, ne, c, 0, &L->wk_dt);
                    else if (strstr(n, "attn_v.weight")) L->wv = jd_resolve(pv, raw, pend, dt, ne, c, 0, &L->wv_dt);
                    else if (strstr(n, "attn_output.weight")) L->wo = jd_resolve(pv, raw, pend, dt, ne, c, 0, &L->wo_dt);
                    else if (strstr(n, "ffn_gate.weight") && !strstr(n, "ffn_gate_inp")) L->gate = jd_resolve(pv, raw, pend, dt, ne, c, 0, &L->gate_dt);
                    else if (strstr(n, "ffn_up.weight")) L->up = jd_resolve(pv, raw, pend, dt, ne, c, 0, &L->up_dt);
                    else if (strstr(n, "ffn_down.weight")) L->down = jd_resolve(pv, raw, pend, dt, ne, c, 0, &L->down_dt);
                    else if (strstr(n, "attn_norm.weight")) L->attn_norm = jd_resolve(pv, raw, pend, dt, ne, c, 1, &wdt);
                    else if (strstr(n, "ffn_norm.weight")) L->ffn_norm = jd_resolve(pv, raw, pend, dt, ne, c, 1, &wdt);
                }
            }
        }
    }
#undef NEED
#undef RD
    free(ti);
    ti = NULL;
    rc = jd_host_finish(h, rope_override, lora_rank);
    if (rc != JD_OK) goto bail;
    rc = jd_vocab_index_build(h);
    if (rc != JD_OK) goto bail;
    return JD_OK;
bail:
    free(ti);
    jd_host_free(h);
    return rc;
}

void jd_host_free(jd_host_model *h) {
    if (!h) return;
    jd_host_priv *pv = (jd_host_priv *)h->priv;
    if (pv) {
        free(pv->vocab_slot);
        for (int i = 0; i < pv->n_owned; i++) free(pv->owned[i]);
        free(pv->owned);
        if (pv->map) munmap(pv->map, pv->map_size);
        free(pv);
    }
    if (h->vocab_tokens) {
        for (int i = 0; i < h->n_vocab_tokens; i++) free(h->vocab_tokens[i]);
        free(h->vocab_tokens);
    }
    memset(h, 0, sizeof(*h));
}

int jd_host_lora_seed(jd_host_model *h, uint64_t seed, int n_alive, float ab_std, float vote_amp) {
    if (!h || !h->priv || n_alive < 0 || n_alive > JD_MAX_EXPERTS) return JD_EINVAL;
    int rc = jd_host_lora_alloc(h, n_alive);
    if (rc != JD_OK) return rc;
    uint64_t s = jd_splitmix64(seed);
    int D = h->dim, R = h->lora_rank;
    for (int l = 0; l < h->n_layers && l < JD_MAX_LAYERS; l++) {
        for (int i = 0; i < JD_MAX_EXPERTS * D; i++) h->w_vote[l][i] = (2.0f * jd_uni(&s) - 1.0f) * vote_amp;
        for (int e = 0; e < JD_MAX_EXPERTS; e++) {
            if (e < n_alive) {
                for (int j = 0; j < D * R; j++) h->A[l][e][j] = jd_normal(&s) * ab_std;
                for (int j = 0; j < R * D; j++) h->B[l][e][j] = jd_normal(&s) * ab_std;
                h->alive[l][e] = 1;
            } else h->alive[l][e] = 0;
        }
    }
    return JD_OK;
}

int jd_host_lora_save(const jd_host_model *h, const char *path) {
    if (!h || !path) return JD_EINVAL;
    FILE *f = fopen(path, "wb");
    if (!f) return JD_EIO;
    int L = h->n_layers < JD_MAX_LAYERS ? h->n_layers : JD_MAX_LAYERS, D = h->dim, R = h->lora_rank, E = JD_MAX_EXPERTS;
    int ok = fwrite("JDLORA01", 1, 8, f) == 8 && w32(f, L) && w32(f, D) && w32(f, R) && w32(f, E);
    for (int l = 0; l < L && ok; l++) for (int e = 0; e < E && ok; e++) ok = w32(f, (uint32_t)h->alive[l][e]);
    for (int l = 0; l < L && ok; l++) ok = fwrite(h->w_vote[l], 4, (size_t)E * D, f) == (size_t)E * D;
    for (int l = 0; l < L && ok; l++)
        for (int e = 0; e < E && ok; e++) {
            if (!h->alive[l][e]) continue;
            ok = fwrite(h->A[l][e], 4, (size_t)D * R, f) == (size_t)D * R && fwrite(h->B[l][e], 4, (size_t)R * D, f) == (size_t)R * D;
        }
    if (fclose(f) != 0) ok = 0;
    return ok ? JD_OK : JD_EIO;
}

int jd_host_lora_load(jd_host_model *h, const char *path) {
    if (!h || !path || !h->priv) return JD_EINVAL;
    FILE *f = fopen(path, "rb");
    if (!f) return JD_EIO;
    char mg[8]; uint32_t L, D, R, E; int rc = JD_EFORMAT;
    if (fread(mg, 1, 8, f) != 8 || memcmp(mg, "JDLORA01", 8) || fread(&L, 4, 1, f) != 1 || fread(&D, 4, 1, f) != 1 ||
        fread(&R, 4, 1, f) != 1 || fread(&E, 4, 1, f) != 1) goto done;
    if ((int)L != (h->n_layers < JD_MAX_LAYERS ? h->n_layers : JD_MAX_LAYERS) || (int)D != h->dim || (int)R != h->lora_rank || E != JD_MAX_EXPERTS) goto done;
    uint32_t alive[JD_MAX_LAYERS][JD_MAX_EXPERTS];
    for (uint32_t l = 0; l < L; l++) if (fread(alive[l], 4, E, f) != E) goto done;
    int n_alive_max = 0;
    for (uint32_t l = 0; l < L; l++) for (uint32_t e = 0; e < E; e++) if (alive[l][e] && (int)e + 1 > n_alive_max) n_alive_max = (int)e + 1;
    if ((rc = jd_host_lora_alloc(h, n_alive_max)) != JD_OK) goto done;
    rc = JD_EFORMAT;
    for (uint32_t l = 0; l < L; l++) if (fread(h->w_vote[l], 4, (size_t)E * D, f) != (size_t)E * D) goto done;
    for (uint32_t l = 0; l < L; l++)
        for (uint32_t e = 0; e < E; e++) {
            h->alive[l][e] = alive[l][e] ? 1 : 0;
            if (!alive[l][e]) continue;
            if (fread(h->A[l][e], 4, (size_t)D * R, f) != (size_t)D * R || fread(h->B[l][e], 4, (size_t)R * D, f) != (size_t)R * D) goto done;
        }
    rc = JD_OK;
done:
    fclose(f);
    return rc;
}

/* ======================= synthetic quantised GGUF ======================= */
/* Q8_0 block of 32 (layout janusdoe.c:2566-2569): f16 d = amax/127, int8 q = round(x/d). */
static void jd_quant_q8_0(const float *x, uint8_t *b) {
    float amax = 0;
    for (int i = 0; i < 32; i++) { float a = fabsf(x[i]); if (a > amax) amax = a; }
    float d = amax / 127.0f, id = d > 0 ? 1.0f / d : 0.0f;
    uint16_t h = jd_f2h(d);
    b[0] = (uint8_t)(h & 0xFF); b[1] = (uint8_t)(h >> 8);
    for (int i = 0; i < 32; i++) { int q = (int)lrintf(x[i] * id); if (q > 127) q = 127; if (q < -127) q = -127; b[2 + i] = (uint8_t)(int8_t)q; }
}
/* Q4_K superblock of 256 (layout janusdoe.c:2554-2561, 2577-2585): 8 sub-blocks of 32 with
 * an affine 4-bit code x ~ d*s_j*q - dmin*m_j; s_j, m_j 6-bit, d and dmin f16. */
static void jd_quant_q4_k(const float *x, uint8_t *b) {
    float sc[8], mn[8], maxsc = 0, maxmn = 0;
    for (int j = 0; j < 8; j++) {
        float lo = 0, hi = 0;
        for (int i = 0; i < 32; i++) { float v = x[32 * j + i]; if (v < lo) lo = v; if (v > hi) hi = v; }
        sc[j] = (hi - lo) / 15.0f; mn[j] = -lo;
        if (sc[j] > maxsc) maxsc = sc[j];
        if (mn[j] > maxmn) maxmn = mn[j];
    }
    uint16_t hd = jd_f2h(maxsc / 63.0f), hm = jd_f2h(maxmn / 63.0f);
    float d = jdq_half(hd), dmin = jdq_half(hm);
    int s6[8], m6[8];
    for (int j = 0; j < 8; j++) {
        int s = d > 0 ? (int)lrintf(sc[j] / d) : 0, m = dmin > 0 ? (int)lrintf(mn[j] / dmin) : 0;
        s6[j] = s < 0 ? 0 : s > 63 ? 63 : s;
        m6[j] = m < 0 ? 0 : m > 63 ? 63 : m;
    }
    b[0] = (uint8_t)(hd & 0xFF); b[1] = (uint8_t)(hd >> 8); b[2] = (uint8_t)(hm & 0xFF); b[3] = (uint8_t)(hm >> 8);
    uint8_t *p = b + 4, *qs = b + 16;
    for (int j = 0; j < 4; j++) {
        p[j] = (uint8_t)((s6[j] & 63) | ((s6[j + 4] >> 4) << 6));
        p[j + 4] = (uint8_t)((m6[j] & 63) | ((m6[j + 4] >> 4) << 6));
        p[j + 8] = (uint8_t)((s6[j + 4] & 15) | ((m6[j + 4] & 15) << 4));
    }
    for (int c = 0; c < 4; c++)
        for (int l = 0; l < 32; l++) {
            int q2[2];
            for (int hh = 0; hh < 2; hh++) {
                int j = 2 * c + hh;
                float step = d * (float)s6[j], off = dmin * (float)m6[j];
                int q = step > 0 ? (int)lrintf((x[64 * c + 32 * hh + l] + off) / step) : 0;
                q2[hh] = q < 0 ? 0 : q > 15 ? 15 : q;
            }
            qs[32 * c + l] = (uint8_t)(q2[0] | (q2[1] << 4));
        }
}

/* Q4_0 / Q5_0 block of 32 (layouts in jd_quant.h): symmetric codes q = round(x/d) + 8 (+16)
 * clamped to 4 (5) bits, d = max|x| / 8 (16) as f16. */
static void jd_quant_q4_0_q5_0(const float *x, uint8_t *b, int five) {
    float amax = 0;
    for (int i = 0; i < 32; i++) if (fabsf(x[i]) > amax) amax = fabsf(x[i]);
    const int bias = five ? 16 : 8, top = five ? 31 : 15;
    uint16_t hd = jd_f2h(amax / (float)bias);
    float d = jdq_half(hd);
    int q[32];
    for (int i = 0; i < 32; i++) {
        int v = d > 0 ? (int)lrintf(x[i] / d) + bias : bias;
        q[i] = v < 0 ? 0 : v > top ? top : v;
    }
    b[0] = (uint8_t)(hd & 0xFF); b[1] = (uint8_t)(hd >> 8);
    uint8_t *nib = b + (five ? 6 : 2);
    if (five) {
        uint32_t fifth = 0;
        for (int i = 0; i < 32; i++) fifth |= (uint32_t)((q[i] >> 4) & 1) << i;
        b[2] = (uint8_t)fifth; b[3] = (uint8_t)(fifth >> 8); b[4] = (uint8_t)(fifth >> 16); b[5] = (uint8_t)(fifth >> 24);
    }
    for (int i = 0; i < 16; i++) nib[i] = (uint8_t)((q[i] & 15) | ((q[i + 16] & 15) << 4));
}
/* Q6_K superblock of 256: 16 groups of 16 with an int8 scale each, d = max|scale|/127 (f16),
 * codes q = round(x/(d*sc)) + 32 in 6 bits, stored as low nibbles + 2-bit high parts. */
static void jd_quant_q6_k(const float *x, uint8_t *b) {
    float gs[16], maxgs = 0;
    for (int g = 0; g < 16; g++) {
        float amax = 0;
        for (int i = 0; i < 16; i++) if (fabsf(x[16 * g + i]) > amax) amax = fabsf(x[16 * g + i]);
        gs[g] = amax / 31.0f;
        if (gs[g] > maxgs) maxgs = gs[g];
    }
    uint16_t hd = jd_f2h(maxgs / 127.0f);
    float d = jdq_half(hd);
    memset(b, 0, 210);
    for (int g = 0; g < 16; g++) {
        int sc = d > 0 ? (int)lrintf(gs[g] / d) : 0;
        sc = sc < -128 ? -128 : sc > 127 ? 127 : sc;
        /* scale index of group g (weights 16g..16g+15): half g/8, quarter (g%8)/2, l0 = 16*(g%2) */
        const int hf = g / 8, u = (g % 8) / 2, li = g % 2;
        b[192 + 8 * hf + li + 2 * u] = (uint8_t)(int8_t)sc;
        const float step = d * (float)sc;
        for (int i = 0; i < 16; i++) {
            int q = step != 0 ? (int)lrintf(x[16 * g + i] / step) + 32 : 32;
            q = q < 0 ? 0 : q > 63 ? 63 : q;
            const int l = 16 * li + i, e = 128 * hf + 32 * u + l;  /* e == 16*g + i */
            (void)e;
            const int qlb = 64 * hf + l + 32 * (u & 1);
            b[qlb] |= (uint8_t)((q & 15) << (4 * (u >> 1)));
            b[128 + 32 * hf + l] |= (uint8_t)(((q >> 4) & 3) << (2 * u));
        }
    }
    b[208] = (uint8_t)(hd & 0xFF); b[209] = (uint8_t)(hd >> 8);
}

typedef struct {
    uint8_t *dst; uint64_t n_chunks; int dt; uint64_t seed; float std; int ti;
    uint64_t next; pthread_mutex_t *mu;
} jd_gen_job;

/* Chunk = 256 elements, normals from state splitmix64(seed ^ ti<<44 ^ chunk), both
 * Box-Muller branches. */
static void jd_gen_chunk(const jd_gen_job *j, uint64_t ch) {
    float x[256];
    uint64_t s = jd_splitmix64(j->seed ^ ((uint64_t)j->ti << 44) ^ (ch * 0x9E3779B97F4A7C15ULL));
    for (int i = 0; i < 256; i += 2) {
        float u1 = jd_uni(&s), u2 = jd_uni(&s);
        if (u1 < 1e-10f) u1 = 1e-10f;
        float r = sqrtf(-2.0f * logf(u1)), a = 6.2831853f * u2;
        x[i] = r * cosf(a) * j->std; x[i + 1] = r * sinf(a) * j->std;
    }
    if (j->dt == JD_Q8_0) for (int b = 0; b < 8; b++) jd_quant_q8_0(x + 32 * b, j->dst + (ch * 8 + b) * 34);
    else if (j->dt == JD_Q4_0) for (int b = 0; b < 8; b++) jd_quant_q4_0_q5_0(x + 32 * b, j->dst + (ch * 8 + b) * 18, 0);
    else if (j->dt == JD_Q5_0) for (int b = 0; b < 8; b++) jd_quant_q4_0_q5_0(x + 32 * b, j->dst + (ch * 8 + b) * 22, 1);
    else if (j->dt == JD_Q4_K) jd_quant_q4_k(x, j->dst + ch * 144);
    else if (j->dt == JD_Q6_K) jd_quant_q6_k(x, j->dst + ch * 210);
    else if (j->dt == JD_F16) for (int i = 0; i < 256; i++) {
        uint16_t h = jd_f2h(x[i]);
        j->dst[ch * 512 + 2 * i] = (uint8_t)(h & 0xFF); j->dst[ch * 512 + 2 * i + 1] = (uint8_t)(h >> 8);
    }
    else memcpy(j->dst + ch * 1024, x, 1024);
}
static void *jd_gen_worker(void *a) {
    jd_gen_job *j = (jd_gen_job *)a;
    for (;;) {
        pthread_mutex_lock(j->mu);
        uint64_t c0 = j->next; j->next += 1024;
        pthread_mutex_unlock(j->mu);
        if (c0 >= j->n_chunks) break;
        uint64_t c1 = c0 + 1024 < j->n_chunks ? c0 + 1024 : j->n_chunks;
        for (uint64_t c = c0; c < c1; c++) jd_gen_chunk(j, c);
    }
    return NULL;
}
static void jd_gen_tensor(uint8_t *dst, uint64_t n, int dt, uint64_t seed, float std, int ti, int threads) {
    pthread_mutex_t mu = PTHREAD_MUTEX_INITIALIZER;
    jd_gen_job job = {dst, n / 256, dt, seed, std, ti, 0, &mu};
    int nt = threads;
    if (nt <= 0) { long c = sysconf(_SC_NPROCESSORS_ONLN); nt = c > 0 ? (int)c : 1; }
    if (nt > 128) nt = 128;
    if ((uint64_t)nt > job.n_chunks / 1024 + 1) nt = (int)(job.n_chunks / 1024 + 1);
    pthread_t th[128];
    int started = 0;
    for (int t = 1; t < nt; t++) if (pthread_create(&th[started], NULL, jd_gen_worker, &job) == 0) started++;
    jd_gen_worker(&job);
    for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
}

/* Text of token id of the synthetic vocabulary: 0-2 "<unk>" "<s>" "</s>", 3-97 the printable
 * ASCII characters, then pseudo-words (syllables of the base-20 digits of n) as "Ġword"
 * (even offsets) and "word" (odd offsets); every id with id % 997 == 500 repeats the text of
 * id - 400, so lookups must return the lowest id of a text. */
static void jd_synth_token(int id, char *buf, size_t cap) {
    static const char *syl[20] = {"a", "e", "i", "o", "u", "ka", "ne", "ri", "so", "tu",
                                  "ma", "le", "pi", "do", "gu", "sh", "th", "ch", "qu", "x"};
    if (id >= 500 && id % 997 == 500) { jd_synth_token(id - 400, buf, cap); return; }
    if (id < 3) { snprintf(buf, cap, "%s", id == 0 ? "<unk>" : id == 1 ? "<s>" : "</s>"); return; }
    if (id < 98) { snprintf(buf, cap, "%c", (char)(32 + id - 3)); return; }
    const int j = id - 98;
    size_t o = 0;
    if ((j & 1) == 0) { buf[o++] = (char)0xC4; buf[o++] = (char)0xA0; }
    char digits[16];
    int nd = 0;
    for (unsigned n = (unsigned)(j / 2 + 1); n; n /= 20) digits[nd++] = (char)(n % 20);
    while (nd-- > 0 && o + 3 < cap) {
        const char *sy = syl[(int)digits[nd]];
        while (*sy && o + 1 < cap) buf[o++] = *sy++;
    }
    buf[o] = '\0';
}

int jd_gguf_write_synthetic(const char *path, const char *arch, int n_layers, int dim, int hidden, int n_heads,
                            int n_kv_heads, int vocab, float rope_theta, float rms_eps, int dtype, uint64_t seed,
                            float std, int threads) {
    return jd_gguf_write_synthetic_mixed(path, arch, n_layers, dim, hidden, n_heads, n_kv_heads, vocab, rope_theta,
                                         rms_eps, dtype, dtype, seed, std, threads);
}

static int jd_synth_dtype_ok(int dt) {
    return dt == JD_F32 || dt == JD_F16 || dt == JD_Q4_0 || dt == JD_Q5_0 || dt == JD_Q8_0 || dt == JD_Q4_K ||
           dt == JD_Q6_K;
}

int jd_gguf_write_synthetic_mixed(const char *path, const char *arch, int n_layers, int dim, int hidden, int n_heads,
                                  int n_kv_heads, int vocab, float rope_theta, float rms_eps, int dtype, int out_dtype,
                                  uint64_t seed, float std, int threads) {
    if (!path || !arch || n_layers < 1 || n_layers > JD_MAX_LAYERS || dim < 1 || n_heads < 1 || n_kv_heads < 1 ||
        n_heads % n_kv_heads || dim % n_heads || vocab < 1 || hidden < 1)
        return JD_EINVAL;
    if (!jd_synth_dtype_ok(dtype) || !jd_synth_dtype_ok(out_dtype)) return JD_EUNSUPPORTED;
    int hd = dim / n_heads, qd = n_heads * hd, kd = n_kv_heads * hd;
    if (dim % 256 || hidden % 256 || qd % 256) return JD_EINVAL;
    int nt = 2 + 1 + 9 * n_layers;
    struct { char name[96]; uint64_t d0, d1; int nd, dt; uint64_t off, bytes; } *t = calloc(nt, sizeof(*t));
    if (!t) return JD_ENOMEM;
    int n = 0;
#define T2(nm, c, r, dtp) do { snprintf(t[n].name, 96, "%s", nm); t[n].d0 = (c); t[n].d1 = (r); t[n].nd = 2; t[n].dt = (dtp); n++; } while (0)
#define T1(nm, c) do { snprintf(t[n].name, 96, "%s", nm); t[n].d0 = (c); t[n].d1 = 1; t[n].nd = 1; t[n].dt = JD_F32; n++; } while (0)
    T2("token_embd.weight", dim, vocab, dtype);
    T1("output_norm.weight", dim);
    T2("output.weight", dim, vocab, out_dtype);
    char nm[96];
    for (int l = 0; l < n_layers; l++) {
        snprintf(nm, 96, "blk.%d.attn_norm.weight", l); T1(nm, dim);
        snprintf(nm, 96, "blk.%d.attn_q.weight", l); T2(nm, dim, qd, dtype);
        snprintf(nm, 96, "blk.%d.attn_k.weight", l); T2(nm, dim, kd, dtype);
        snprintf(nm, 96, "blk.%d.attn_v.weight", l); T2(nm, dim, kd, dtype);
        snprintf(nm, 96, "blk.%d.attn_output.weight", l); T2(nm, qd, dim, dtype);
        snprintf(nm, 96, "blk.%d.ffn_norm.weight", l); T1(nm, dim);
        snprintf(nm, 96, "blk.%d.ffn_gate.weight", l); T2(nm, dim, hidden, dtype);
        snprintf(nm, 96, "blk.%d.ffn_up.weight", l); T2(nm, dim, hidden, dtype);
        snprintf(nm, 96, "blk.%d.ffn_down.weight", l); T2(nm, hidden, dim, dtype);
    }
#undef T1
#undef T2
    uint64_t off = 0;
    for (int i = 0; i < n; i++) {
        t[i].off = off;
        t[i].bytes = jdq_bytes(t[i].dt, t[i].d0 * t[i].d1);
        off += (t[i].bytes + 31) / 32 * 32;
    }
    FILE *f = fopen(path, "wb");
    if (!f) { free(t); return JD_EIO; }
    char k[128];
    int ok = w32(f, 0x46554747) && w32(f, 3) && w64(f, (uint64_t)n) && w64(f, 13);
    ok = ok && wkv_s(f, "general.architecture", arch);
    snprintf(k, 128, "%s.embedding_length", arch); ok = ok && wkv_u(f, k, dim);
    snprintf(k, 128, "%s.block_count", arch); ok = ok && wkv_u(f, k, n_layers);
    snprintf(k, 128, "%s.attention.head_count", arch); ok = ok && wkv_u(f, k, n_heads);
    snprintf(k, 128, "%s.attention.head_count_kv", arch); ok = ok && wkv_u(f, k, n_kv_heads);
    snprintf(k, 128, "%s.feed_forward_length", arch); ok = ok && wkv_u(f, k, hidden);
    snprintf(k, 128, "%s.vocab_size", arch); ok = ok && wkv_u(f, k, vocab);
    snprintf(k, 128, "%s.rope.freq_base", arch); ok = ok && wkv_f(f, k, rope_theta);
    snprintf(k, 128, "%s.attention.layer_norm_rms_epsilon", arch); ok = ok && wkv_f(f, k, rms_eps);
    snprintf(k, 128, "%s.context_length", arch); ok = ok && wkv_u(f, k, 4096);
    ok = ok && wkv_u(f, "tokenizer.ggml.bos_token_id", 1) && wkv_u(f, "tokenizer.ggml.eos_token_id", 2);
    ok = ok && wstr(f, "tokenizer.ggml.tokens") && w32(f, 9) && w32(f, 8) && w64(f, (uint64_t)vocab);
    for (int id = 0; id < vocab && ok; id++) {
        char tb[64];
        jd_synth_token(id, tb, sizeof tb);
        ok = wstr(f, tb);
    }
    for (int i = 0; i < n && ok; i++) {
        ok = wstr(f, t[i].name) && w32(f, t[i].nd) && w64(f, t[i].d0);
        if (t[i].nd == 2) ok = ok && w64(f, t[i].d1);
        ok = ok && w32(f, t[i].dt) && w64(f, t[i].off);
    }
    long p = ftell(f), al = ((p + 31) / 32) * 32;
    for (long i = p; i < al && ok; i++) ok = fputc(0, f) != EOF;
    uint8_t *buf = NULL;
    for (int i = 0; i < n && ok; i++) {
        uint64_t padded = (t[i].bytes + 31) / 32 * 32;
        uint8_t *nb = realloc(buf, padded);
        if (!nb) { ok = 0; break; }
        buf = nb;
        memset(buf + t[i].bytes, 0, padded - t[i].bytes);
        if (t[i].nd == 1) { for (uint64_t j = 0; j < t[i].d0; j++) ((float *)buf)[j] = 1.0f; }
        else jd_gen_tensor(buf, t[i].d0 * t[i].d1, t[i].dt, seed, std, i, threads);
        ok = fwrite(buf, 1, padded, f) == padded;
    }
    free(buf);
    if (fclose(f) != 0) ok = 0;
    free(t);
    return ok ? JD_OK : JD_EIO;
}

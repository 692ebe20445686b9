/*
 * ref_harness.c — drives the reference's own code (TEST INFRASTRUCTURE ONLY).
 *
 * The reference is one C translation unit whose functions are all `static`.  This
 * harness compiles that unmodified source into the same unit (its `main` renamed)
 * and exports a small C interface over the functions on the decode path, so the
 * oracle restatement can be pinned against the reference itself and golden fixtures
 * can be generated.  oracle/Makefile points JD_REF_SRC at the reference checkout and
 * writes the shared objects to oracle/_ref/ (never committed).
 *
 * Exported state is global (one own model, one host model at a time), like the
 * reference's own globals.
 */
#define main janusdoe_main
#include JD_REF_SRC
#undef main

#define JDR_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------ rng */
static uint64_t jdr_splitmix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    z = z ^ (z >> 31);
    return z ? z : 1;
}
JDR_API void jdr_rng_set(uint64_t s) { rng_state = s; }
JDR_API uint64_t jdr_rng_get(void) { return rng_state; }
JDR_API uint64_t jdr_rng_next(void) { return rng_next(); }
JDR_API float jdr_rand_uniform(void) { return rand_uniform(); }
JDR_API float jdr_rand_normal(void) { return rand_normal(); }
JDR_API int jdr_lora_rank(void) { return LORA_RANK; }

/* ------------------------------------------------------------ own model */
static Config g_c;
static ModelW g_w;
static RunState g_rs;
static int g_have_own = 0;

static void jdr_fill(Tensor *t, float std) { for (int i = 0; i < t->size; i++) t->data[i] = rand_normal() * std; }

/* config_from_depth + overrides, init_weights, then the seeded overwrite:
 * rng_state = splitmix64(seed); tok_emb, output; per layer wq, wk, wv, wo, w_vote;
 * experts 0..initial-1 gate, up, down; optional alive masks from the same stream. */
JDR_API int jdr_own_setup(int depth, int n_kv_heads, int vocab, int seq_len, uint64_t seed, float std, int draw_masks) {
    g_c = config_from_depth(depth);
    if (n_kv_heads > 0) g_c.n_kv_heads = n_kv_heads;
    g_c.vocab_size = vocab;
    g_c.seq_len = seq_len;
    rng_state = 42;
    init_weights(&g_w, &g_c);
    rng_state = jdr_splitmix64(seed);
    jdr_fill(g_w.tok_emb, std); jdr_fill(g_w.output, std);
    for (int l = 0; l < g_c.depth; l++) {
        LayerW *lw = &g_w.layers[l];
        jdr_fill(lw->wq, std); jdr_fill(lw->wk, std); jdr_fill(lw->wv, std); jdr_fill(lw->wo, std);
        jdr_fill(lw->parliament.w_vote, std);
        for (int e = 0; e < g_c.initial_experts; e++) {
            jdr_fill(lw->experts[e].w_gate, std); jdr_fill(lw->experts[e].w_up, std); jdr_fill(lw->experts[e].w_down, std);
        }
    }
    if (draw_masks) {
        int n0 = g_c.initial_experts, lo = n0 - 3 < MIN_EXPERTS ? MIN_EXPERTS : n0 - 3;
        for (int l = 0; l < g_c.depth; l++) {
            LayerW *lw = &g_w.layers[l];
            int target = lo + (int)(rng_next() % (uint64_t)(n0 - lo + 1));
            while (lw->n_alive > target) {
                int e = (int)(rng_next() % (uint64_t)n0);
                if (lw->experts[e].alive) { free_expert(&lw->experts[e]); lw->n_alive--; }
            }
        }
    }
    g_rs = alloc_run(&g_c);
    g_have_own = 1;
    return 0;
}
JDR_API int jdr_own_dims(int *out) {
    out[0] = g_c.depth; out[1] = g_c.dim; out[2] = g_c.n_heads; out[3] = g_c.n_kv_heads; out[4] = g_c.head_dim;
    out[5] = g_c.hidden_dim; out[6] = g_c.vocab_size; out[7] = g_c.seq_len; out[8] = g_c.initial_experts;
    return 0;
}
JDR_API int jdr_own_alive(int l, int *alive16) {
    for (int e = 0; e < MAX_EXPERTS; e++) alive16[e] = g_w.layers[l].experts[e].alive;
    return g_w.layers[l].n_alive;
}
/* copy a weight tensor out: which = 0 tok_emb, 1 output, 2 wq, 3 wk, 4 wv, 5 wo, 6 w_vote, 7 gate, 8 up, 9 down */
JDR_API int jdr_own_tensor(int which, int l, int e, float *out, long n) {
    Tensor *t = NULL;
    switch (which) {
    case 0: t = g_w.tok_emb; break; case 1: t = g_w.output; break;
    case 2: t = g_w.layers[l].wq; break; case 3: t = g_w.layers[l].wk; break;
    case 4: t = g_w.layers[l].wv; break; case 5: t = g_w.layers[l].wo; break;
    case 6: t = g_w.layers[l].parliament.w_vote; break;
    case 7: t = g_w.layers[l].experts[e].w_gate; break; case 8: t = g_w.layers[l].experts[e].w_up; break;
    case 9: t = g_w.layers[l].experts[e].w_down; break;
    }
    if (!t || t->size != n) return -1;
    memcpy(out, t->data, (size_t)n * 4);
    return 0;
}
/* new sequence: zero the caches (janusdoe.c chat) and restart every EMA at 0.5 */
JDR_API void jdr_own_reset_seq(void) {
    int kd = g_c.n_kv_heads * g_c.head_dim;
    memset(g_rs.key_cache, 0, (size_t)g_c.depth * g_c.seq_len * kd * 4);
    memset(g_rs.value_cache, 0, (size_t)g_c.depth * g_c.seq_len * kd * 4);
    for (int l = 0; l < g_c.depth; l++) g_w.layers[l].parliament.consensus = 0.5f;
}
JDR_API int jdr_own_forward(int token, int pos, float *logits, float *ema) {
    float *lg = forward_token(&g_w, &g_c, &g_rs, token, pos);
    memcpy(logits, lg, (size_t)g_c.vocab_size * 4);
    if (ema) for (int l = 0; l < g_c.depth; l++) ema[l] = g_w.layers[l].parliament.consensus;
    return 0;
}
JDR_API int jdr_own_export(const char *path) {
    snprintf(g_c.gguf_path, sizeof(g_c.gguf_path), "%s", path);
    export_gguf(&g_w, &g_c);
    return 0;
}
/* load_own_gguf into a freshly initialised model of the same config */
JDR_API int jdr_own_load(const char *path) { return load_own_gguf(path, &g_w, &g_c); }

/* sample() with an explicit RNG state (in/out) */
JDR_API int jdr_sample(float *logits, int V, float temp, int top_k, uint64_t *state) {
    uint64_t save = rng_state; rng_state = *state;
    int r = sample(logits, V, temp, top_k);
    *state = rng_state; rng_state = save;
    return r;
}

/* -------------------------------------------------------- packed quant */
JDR_API float jdr_f16_to_f32(uint16_t h) { return jd_f16_to_f32(h); }
JDR_API int jdr_dequant(const uint8_t *src, float *out, uint64_t n, int dt) { return jd_dequant_any(src, out, n, dt); }
JDR_API int jdr_qmatvec(float *out, const uint8_t *W, int dt, const float *x, int r, int c) { return jd_qmatvec(out, W, dt, x, r, c); }

/* ------------------------------------------------------------ host mode */
static GGUFHost g_h;
static float *g_kc = NULL, *g_vc = NULL;
static int g_max_seq = 0;

JDR_API int jdr_host_load(const char *path, int rope_override) {
    g_rope_override = rope_override;
    rng_state = 42;
    return gguf_host_load(&g_h, path, 0);
}
JDR_API int jdr_host_dims(int *out) {
    out[0] = g_h.host_n_layers; out[1] = g_h.host_dim; out[2] = g_h.host_hidden; out[3] = g_h.host_heads;
    out[4] = g_h.host_kv_heads; out[5] = g_h.host_head_dim; out[6] = g_h.host_vocab; out[7] = host_rope_norm(&g_h);
    out[8] = g_h.host_output_dt; out[9] = g_h.host_bos; out[10] = g_h.host_eos;
    return 0;
}
JDR_API float jdr_host_theta(void) { return g_h.rope_theta; }
JDR_API float jdr_host_eps(void) { return g_h.rms_eps; }
/* Synthetic LoRA parliament (same scheme as the oracle): state = splitmix64(seed); per
 * layer 16 vote rows uniform (2u-1)*amp, then experts e < n_alive draw A then B as
 * rand_normal()*std; experts >= n_alive are dead. */
JDR_API int jdr_host_lora_seed(uint64_t seed, int n_alive, float ab_std, float vote_amp) {
    rng_state = jdr_splitmix64(seed);
    int D = g_h.host_dim;
    for (int l = 0; l < g_h.host_n_layers && l < LORA_MAX_LAYERS; l++) {
        for (int i = 0; i < MAX_EXPERTS * D; i++) g_h.w_vote[l][i] = (2.0f * rand_uniform() - 1.0f) * vote_amp;
        for (int e = 0; e < MAX_EXPERTS; e++) {
            HostExpert *ex = &g_h.experts[l][e];
            if (e < n_alive) {
                if (!ex->A) ex->A = calloc((size_t)D * LORA_RANK, 4);
                if (!ex->B) ex->B = calloc((size_t)LORA_RANK * D, 4);
                if (!ex->A || !ex->B) return -1;
                for (int j = 0; j < D * LORA_RANK; j++) ex->A[j] = rand_normal() * ab_std;
                for (int j = 0; j < LORA_RANK * D; j++) ex->B[j] = rand_normal() * ab_std;
                ex->alive = 1;
            } else ex->alive = 0;
        }
    }
    return 0;
}
JDR_API int jdr_host_reset_seq(int max_seq) {
    int kd = g_h.host_kv_heads * g_h.host_head_dim;
    if (max_seq != g_max_seq) {
        free(g_kc); free(g_vc);
        g_kc = calloc((size_t)g_h.host_n_layers * max_seq * kd, 4);
        g_vc = calloc((size_t)g_h.host_n_layers * max_seq * kd, 4);
        g_max_seq = max_seq;
        if (!g_kc || !g_vc) return -1;
    } else {
        memset(g_kc, 0, (size_t)g_h.host_n_layers * max_seq * kd * 4);
        memset(g_vc, 0, (size_t)g_h.host_n_layers * max_seq * kd * 4);
    }
    for (int l = 0; l < g_h.host_n_layers && l < LORA_MAX_LAYERS; l++) g_h.consensus[l] = 0.5f;
    return 0;
}
JDR_API int jdr_host_forward(int token, int pos, float *logits, float *ema) {
    gguf_host_forward(&g_h, token, pos, logits, g_kc, g_vc, g_max_seq);
    if (ema) for (int l = 0; l < g_h.host_n_layers && l < LORA_MAX_LAYERS; l++) ema[l] = g_h.consensus[l];
    return 0;
}
/* host_learn_run (janusdoe.c:3420) with the global RNG state and notorch offset set from /
 * returned to the caller; caches of max_seq positions */
JDR_API int jdr_host_learn(const int *toks, int nt, int max_seq, float lr, uint64_t *rng, int *offset) {
    rng_state = *rng;
    host_notorch_offset = *offset;
    int d = host_learn_run(&g_h, toks, nt, max_seq, lr);
    *rng = rng_state;
    *offset = host_notorch_offset;
    return d;
}
/* expert (l, e)'s LoRA factors A [D][R], B [R][D] and its alive flag */
JDR_API int jdr_host_expert(int l, int e, float *A, float *B) {
    HostExpert *ex = &g_h.experts[l][e];
    if (ex->A && A) memcpy(A, ex->A, (size_t)g_h.host_dim * LORA_RANK * 4);
    if (ex->B && B) memcpy(B, ex->B, (size_t)g_h.host_dim * LORA_RANK * 4);
    return ex->alive;
}
/* host_tokenize on the loaded vocabulary (janusdoe.c:3334) */
JDR_API int jdr_host_tokenize(const char *text, int *out, int max) { return host_tokenize(&g_h, text, out, max); }
/* host_decode_print (janusdoe.c:3348) captured from stdout into buf (NUL-terminated) */
JDR_API int jdr_host_decode_print(int id, char *buf, int cap) {
    fflush(stdout);
    FILE *saved = stdout, *mem = fmemopen(buf, (size_t)cap, "w");
    if (!mem) return -1;
    stdout = mem;
    host_decode_print(&g_h, id);
    fflush(mem);
    long n = ftell(mem);
    stdout = saved;
    fclose(mem);
    if (n >= cap) n = cap - 1;
    buf[n] = '\0';
    return (int)n;
}
JDR_API void jdr_host_free(void) {
    gguf_host_free(&g_h);
    free(g_kc); free(g_vc); g_kc = g_vc = NULL; g_max_seq = 0;
}

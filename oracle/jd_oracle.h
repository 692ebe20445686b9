/*
 * jd_oracle.h — CPU restatement of the janus.DoE decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the parity oracle: plain C99, single
 * precision, the same operation order as the reference so that it reproduces
 * the reference bit for bit when both are built with the same compiler flags.
 * Only the tests, the smoke check and the CPU-baseline leg of the benchmark
 * may load it.  The product path never links or calls anything here.
 *
 * Every function cites the reference function it restates as
 * janusdoe.c:<line>.  Parity pin: tests compare this oracle against the
 * reference source itself, compiled by oracle/Makefile into oracle/_ref/
 * (see ref_harness.c), and against the committed fixtures in tests/golden/
 * that were produced by that build.
 */
#ifndef JD_ORACLE_H
#define JD_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#define JDO_MAX_EXPERTS 16   /* janusdoe.c:116 MAX_EXPERTS */
#define JDO_MAX_LAYERS 32    /* janusdoe.c:117 MAX_LAYERS, janusdoe.c:2533 LORA_MAX_LAYERS */
#define JDO_MIN_EXPERTS 2    /* janusdoe.c:118 */

#ifdef __cplusplus
extern "C" {
#endif

/* ---- RNG (janusdoe.c:190-193) ------------------------------------------ */
uint64_t jdo_splitmix64(uint64_t x);       /* seed -> xorshift state (never 0) */
uint64_t jdo_rng_next(uint64_t *s);        /* janusdoe.c:191 */
float    jdo_rand_uniform(uint64_t *s);    /* janusdoe.c:192 */
float    jdo_rand_normal(uint64_t *s);     /* janusdoe.c:193 */

/* ---- own model ---------------------------------------------------------- */
typedef struct {                            /* janusdoe.c:136-149 (decode fields) */
    int depth, dim, n_heads, n_kv_heads, head_dim, hidden_dim, vocab_size, seq_len;
    float norm_eps, rope_theta, attn_clamp;
    int active_depth, initial_experts;
} jdo_config;

typedef struct {                            /* janusdoe.c:708-713 LayerW + Parliament */
    float *attn_norm, *ffn_norm, *wq, *wk, *wv, *wo, *w_vote;
    float *w_gate[JDO_MAX_EXPERTS], *w_up[JDO_MAX_EXPERTS], *w_down[JDO_MAX_EXPERTS];
    int alive[JDO_MAX_EXPERTS];
    float consensus;                        /* EMA value a fresh sequence starts from */
    float temperature;                      /* Parliament.temperature, 0 on a fresh model */
} jdo_layer;

typedef struct {                            /* janusdoe.c:715-719 ModelW */
    jdo_config c;
    float *tok_emb, *output, *output_norm;
    jdo_layer layers[JDO_MAX_LAYERS];
} jdo_own;

typedef struct {                            /* janusdoe.c:845-851 RunState + per-sequence EMA */
    float *key_cache, *value_cache, *cos_cache, *sin_cache;
    float consensus[JDO_MAX_LAYERS];
    float *x, *xb, *xb2, *hb, *hb2, *q, *k, *v, *att, *logits, *expert_out;
} jdo_own_state;

typedef struct {                            /* one election: what parliament_elect returns */
    int k, n_alive;
    int sel[JDO_MAX_EXPERTS];
    float w[JDO_MAX_EXPERTS];
    float votes[JDO_MAX_EXPERTS];           /* by expert slot */
    float ema;                              /* consensus after the update */
} jdo_elect;

int  jdo_config_from_depth(int depth, jdo_config *c);                      /* janusdoe.c:151-185 */
int  jdo_own_alloc(jdo_own *m, const jdo_config *c);                       /* janusdoe.c:744-776 shapes */
void jdo_own_fill_seeded(jdo_own *m, uint64_t seed, float std, int draw_masks);
void jdo_own_free(jdo_own *m);
int  jdo_own_state_alloc(const jdo_own *m, jdo_own_state *s);              /* janusdoe.c:853-877 */
void jdo_own_state_reset(const jdo_own *m, jdo_own_state *s);
void jdo_own_state_free(jdo_own_state *s);
int  jdo_parliament_elect(const jdo_layer *lw, float *consensus, const float *in, int dim,
                          int *selected, float *weights, jdo_elect *trace); /* janusdoe.c:779-838 */
const float *jdo_own_forward(const jdo_own *m, jdo_own_state *s, int token, int pos,
                             jdo_elect *trace);                            /* janusdoe.c:879-934 */
int  jdo_sample(float *logits, int V, float temp, int top_k, uint64_t *rng); /* janusdoe.c:3637-3645 */
int  jdo_argmax(const float *logits, int V);
void jdo_prompt(uint64_t seq_seed, int V, int n, int *out, uint64_t *rng_after);

/* ---- packed quant (janusdoe.c:2545-2694) --------------------------------- */
float    jdo_f16_to_f32(uint16_t h);                                        /* janusdoe.c:2545 */
uint64_t jdo_quant_bytes(int dt, uint64_t n);                               /* janusdoe.c:2597 */
int      jdo_dequant(const uint8_t *src, float *out, uint64_t n, int dt);  /* janusdoe.c:2602 */
int      jdo_qmatvec(float *out, const uint8_t *W, int dt, const float *x, int r, int c); /* janusdoe.c:2685 */
void     jdo_matvec(float *out, const float *W, const float *x, int r, int c);            /* janusdoe.c:505-519 */
void     jdo_set_threads(int n);

/* ---- host GGUF model ------------------------------------------------------ */
typedef struct {                            /* janusdoe.c:2764-2800 GGUFHost (decode fields) */
    int n_layers, dim, hidden, n_heads, n_kv_heads, head_dim, vocab;
    float rope_theta, rms_eps;
    int rope_norm;                          /* 1 NORM (2i,2i+1), 0 NEOX (i,i+hd/2) */
    char arch[64];
    int bos, eos;
    uint8_t *map; size_t map_size;
    float *tok_emb;                         /* dequantized [V][D] */
    const void *output; int output_dt;
    float *output_norm;
    struct {
        const void *wq, *wk, *wv, *wo, *gate, *up, *down;
        int wq_dt, wk_dt, wv_dt, wo_dt, gate_dt, up_dt, down_dt;
        float *attn_norm, *ffn_norm;
    } layers[JDO_MAX_LAYERS];
    float *dq[JDO_MAX_LAYERS * 3 + 4]; int n_dq;
    int lora_rank; float lora_alpha;
    float *w_vote[JDO_MAX_LAYERS];          /* [16][D] */
    float *A[JDO_MAX_LAYERS][JDO_MAX_EXPERTS], *B[JDO_MAX_LAYERS][JDO_MAX_EXPERTS];
    int alive[JDO_MAX_LAYERS][JDO_MAX_EXPERTS];
    float consensus0[JDO_MAX_LAYERS], attention_bias[JDO_MAX_LAYERS], layer_focus[JDO_MAX_LAYERS];
} jdo_host;

typedef struct {
    int max_seq;
    float *kc, *vc;                         /* [L][max_seq][kd] */
    float consensus[JDO_MAX_LAYERS];
    float *host_x, *host_dy;                /* learning captures of the last forward (janusdoe.c:3274, 3311) */
    int tokens_seen[JDO_MAX_LAYERS][JDO_MAX_EXPERTS];
} jdo_host_state;

int  jdo_rope_norm_for_arch(const char *arch);                              /* janusdoe.c:3153-3156 */
int  jdo_host_load(jdo_host *h, const char *path, int rope_override, int lora_rank); /* janusdoe.c:2837-3048 */
void jdo_host_lora_seed(jdo_host *h, uint64_t seed, int n_alive, float ab_std, float vote_amp);
void jdo_host_free(jdo_host *h);                                            /* janusdoe.c:3449-3467 */
int  jdo_host_state_alloc(const jdo_host *h, jdo_host_state *s, int max_seq);
void jdo_host_state_reset(const jdo_host *h, jdo_host_state *s);
void jdo_host_state_free(jdo_host_state *s);
int  jdo_host_elect(const jdo_host *h, int l, float *consensus, const float *xn, int D,
                    int *selected, float *weights, jdo_elect *trace);      /* janusdoe.c:3054-3087 */
void jdo_host_forward(const jdo_host *h, jdo_host_state *s, int token, int pos,
                      float *logits, jdo_elect *trace);                     /* janusdoe.c:3160-3322 */
/* Hebbian adaptation pass over a token stream (janusdoe.c:3416-3447): per token a forward
 * from position 0 of fresh caches, the prophecy-debt signal of the next token, a notorch
 * step on every expert elected in that token, quarantine.  The reference's global RNG state
 * and notorch offset are explicit here (in/out).  Returns the experts killed. */
int  jdo_host_learn_run(jdo_host *h, jdo_host_state *s, const int *toks, int nt, float lr,
                        uint64_t *rng, int *notorch_offset);

#ifdef __cplusplus
}
#endif
#endif

/*
 * jdgpu.h — C ABI of the B200 decode engine for janus.DoE.
 *
 * Two groups of entry points:
 *   jd_*   host-side model code: the reference's structs, weight generation and GGUF
 *          formats (no CUDA).  These replace the reference's Config / ModelW / GGUFHost
 *          handling (janusdoe.c:136-185, 703-776, 1781-1961, 2745-3048).
 *   jdg_*  the GPU engine: upload a model, then run decode steps on sm_100a kernels.
 *          These replace the reference's token loop (forward_token janusdoe.c:879,
 *          parliament_elect janusdoe.c:779, sample janusdoe.c:3637, gguf_host_forward
 *          janusdoe.c:3160, host_parliament_elect janusdoe.c:3054, jd_qmatvec
 *          janusdoe.c:2685).
 *
 * Conventions: every call returns an int status (JD_OK = 0, negative on error) and
 * never aborts; jdg_last_error() describes the last failure on a context.  All pointer
 * arguments are host pointers unless the name ends in _dev.  One host thread drives a
 * context; each engine owns its device buffers and runs on its own CUDA stream.
 */
#ifndef JDGPU_H
#define JDGPU_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define JD_MAX_EXPERTS 16 /* janusdoe.c:116 */
#define JD_MAX_LAYERS 32  /* janusdoe.c:117, 2533 */

enum {
    JD_OK = 0,
    JD_EINVAL = -1,       /* bad argument or shape */
    JD_ENOMEM = -2,       /* host or device allocation failed */
    JD_ECUDA = -3,        /* a CUDA call failed */
    JD_EFORMAT = -4,      /* malformed or truncated file */
    JD_EUNSUPPORTED = -5, /* packed dtype without a kernel (janusdoe.c:2739 aborts here) */
    JD_EIO = -6,          /* open/read/write failed */
    JD_ESTATE = -7,       /* call out of order, or device-side check failed */
    JD_ECOMM = -8         /* NCCL failure */
};

/* GGUF tensor dtypes used by the host path (janusdoe.c:2543) */
enum { JD_F32 = 0, JD_F16 = 1, JD_Q4_0 = 2, JD_Q5_0 = 6, JD_Q8_0 = 8, JD_Q4_K = 12, JD_Q6_K = 14 };

/* ------------------------------------------------------------------------------------
 * Own model ("organism").  Layout mirrors Config (janusdoe.c:136-149), LayerW +
 * Parliament (janusdoe.c:625-634, 708-713) and ModelW (janusdoe.c:715-719).  Weights are
 * row-major f32 [out][in] as in the reference; dead expert slots have NULL pointers
 * and alive = 0.
 * ---------------------------------------------------------------------------------- */
typedef struct {
    int depth, dim, n_heads, n_kv_heads, head_dim, hidden_dim, vocab_size, seq_len;
    float norm_eps, rope_theta, attn_clamp;
    int active_depth, initial_experts;
} jd_config;

typedef struct {
    float *attn_norm, *ffn_norm, *wq, *wk, *wv, *wo, *w_vote; /* w_vote: [16][dim] */
    float *w_gate[JD_MAX_EXPERTS], *w_up[JD_MAX_EXPERTS], *w_down[JD_MAX_EXPERTS];
    int alive[JD_MAX_EXPERTS];
    float consensus;   /* Parliament.consensus: the EMA a fresh sequence starts from */
    float temperature; /* Parliament.temperature (<= 0.05 means 1) */
} jd_layer;

typedef struct {
    jd_config c;
    float *tok_emb, *output, *output_norm;
    jd_layer layers[JD_MAX_LAYERS];
} jd_model;

/* config_from_depth (janusdoe.c:151-185); vocab_size is set to 258 + merges */
int jd_config_from_depth(int depth, jd_config *c);
/* allocate a model of config c the way init_weights shapes it (janusdoe.c:744-776) */
int jd_model_alloc(jd_model *m, const jd_config *c);
void jd_model_free(jd_model *m);
/* Synthetic weights: xorshift state = splitmix64(seed); every tensor is overwritten with
 * rand_normal()*std (janusdoe.c:190-193) in the order tok_emb, output, then per layer wq,
 * wk, wv, wo, w_vote, experts 0..initial-1 (gate, up, down); norms stay 1.  draw_masks:
 * per layer, a target alive count in [max(2, n-3), n] is drawn and slots are killed. */
int jd_model_fill_seeded(jd_model *m, uint64_t seed, float std, int draw_masks);
/* export_gguf (janusdoe.c:1781-1826): f32, alive experts only */
int jd_model_export_gguf(const jd_model *m, const char *path);
/* load_own_gguf (janusdoe.c:1832-1961): m must be allocated with the file's config;
 * experts present in the file are revived, absent ones are killed. */
int jd_model_load_gguf(jd_model *m, const char *path);

/* ------------------------------------------------------------------------------------
 * Host GGUF model.  Mirrors GGUFHost (janusdoe.c:2764-2800): packed weights point into
 * a read-only mmap, tok_emb and norms are dequantised to f32 at load (janusdoe.c:2817),
 * and the LoRA parliament has per-layer experts A [dim][rank], B [rank][dim].
 * ---------------------------------------------------------------------------------- */
typedef struct {
    const void *wq, *wk, *wv, *wo, *gate, *up, *down;
    int wq_dt, wk_dt, wv_dt, wo_dt, gate_dt, up_dt, down_dt;
    const float *attn_norm, *ffn_norm; /* NULL = all ones */
} jd_host_layer;

typedef struct {
    int n_layers, dim, hidden, n_heads, n_kv_heads, head_dim, vocab;
    float rope_theta, rms_eps;
    int rope_norm; /* 1 NORM (2i,2i+1), 0 NEOX (i,i+hd/2): janusdoe.c:3148-3156 */
    char arch[64];
    int bos, eos;
    const float *tok_emb; /* [vocab][dim] f32 */
    const void *output;
    int output_dt;
    const float *output_norm;
    jd_host_layer layers[JD_MAX_LAYERS];
    int lora_rank;
    float lora_alpha;                                    /* 0.1 (janusdoe.c:2841) */
    float *w_vote[JD_MAX_LAYERS];                        /* [16][dim] */
    float *A[JD_MAX_LAYERS][JD_MAX_EXPERTS];             /* [dim][rank] */
    float *B[JD_MAX_LAYERS][JD_MAX_EXPERTS];             /* [rank][dim] */
    int alive[JD_MAX_LAYERS][JD_MAX_EXPERTS];
    float consensus0[JD_MAX_LAYERS];                     /* 0.5 (janusdoe.c:3026) */
    float attention_bias[JD_MAX_LAYERS], layer_focus[JD_MAX_LAYERS]; /* 0 and 1 */
    char **vocab_tokens; /* tokenizer.ggml.tokens, NULL if absent */
    int n_vocab_tokens;
    void *priv;          /* loader bookkeeping (mmap, dequant buffers) */
} jd_host_model;

/* gguf_host_load (janusdoe.c:2837-3048). rope_override: -1 arch heuristic, 0 NEOX, 1 NORM.
 * The LoRA parliament is allocated with lora_rank and 4 alive zero experts, consensus 0.5. */
int jd_host_load_gguf(jd_host_model *h, const char *path, int rope_override, int lora_rank);
void jd_host_free(jd_host_model *h); /* gguf_host_free (janusdoe.c:3449-3467) */
/* host_tokenize (janusdoe.c:3329-3347): words split at spaces, each looked up as
 * "\xc4\xa0word" then "word" (first 120 bytes), else byte by byte; at most max ids.
 * Returns the number of ids (0 when the file has no vocabulary) or JD_EINVAL. */
int jd_host_tokenize(const jd_host_model *h, const char *text, int *out, int max);
/* host_decode_print (janusdoe.c:3348-3356) into buf: the token's printable form ("Ġ" as a
 * space, "Ċ" as a newline, other non-ASCII bytes dropped; "<id>" for an id without text).
 * Returns the length written (at most cap - 1) or JD_EINVAL. */
int jd_host_token_text(const jd_host_model *h, int id, char *buf, int cap);
/* Synthetic LoRA parliament: state = splitmix64(seed); per layer 16 vote rows uniform
 * (2u-1)*vote_amp, then experts e < n_alive draw A then B as rand_normal()*ab_std. */
int jd_host_lora_seed(jd_host_model *h, uint64_t seed, int n_alive, float ab_std, float vote_amp);
/* LoRA sidecar "JDLORA01": L, D, rank, alive mask, w_vote, A, B (f32 little-endian).
 * The reference re-draws its LoRA at every load; the sidecar lets runs share one. */
int jd_host_lora_save(const jd_host_model *h, const char *path);
int jd_host_lora_load(jd_host_model *h, const char *path);
/* Decode n weights of GGUF type dt (JD_F16, JD_Q4_0, JD_Q5_0, JD_Q8_0, JD_Q4_K, JD_Q6_K; n a
 * whole number of blocks) to f32, bit-identical to the reference's dequantisation
 * (jd_f16_to_f32 and jd_dequant_q4_0/q5_0/q8_0/q4_k/q6_k, janusdoe.c:2545-2596).
 * Returns JD_OK, or JD_EUNSUPPORTED for another type. */
int jd_dequant(const void *src, float *out, uint64_t n, int dt);
/* Tensor-parallel shard of a host model for rank `rank` of `world` (the partition that
 * jdg_host_upload_tp uploads; no counterpart in the single-process reference): query heads
 * [q_head0, q_head0 + q_heads) with their q rows and Wo contraction columns, KV heads
 * [kv_head0, kv_head0 + kv_heads), FFN hidden units [hidden0, hidden0 + hidden) with their
 * gate/up rows and down contraction columns, vocabulary rows [vocab0, vocab0 + vocab).
 * Returns JD_EINVAL when heads, KV heads or hidden units do not divide by world. */
typedef struct {
    int q_head0, q_heads, kv_head0, kv_heads, hidden0, hidden, vocab0, vocab;
} jd_tp_shard;
int jd_tp_shard_of(const jd_host_model *h, int rank, int world, jd_tp_shard *out);
/* Write a synthetic llama-family GGUF v3 (the format gguf_host_load reads): weights
 * N(0, std) quantised per block to dtype (JD_Q8_0 or JD_Q4_K; norms f32 = 1), metadata
 * keys as the loader matches them, BOS 1 / EOS 2 and a synthetic vocabulary of `vocab`
 * tokens (control tokens, the printable ASCII characters, then pseudo-words with and
 * without the "\xc4\xa0" space marker, with some repeated texts).  Tensors are generated
 * in parallel blocks from splitmix64(seed ^ tensor index ^ block index); threads <= 0
 * uses all cores. */
int jd_gguf_write_synthetic(const char *path, const char *arch, int n_layers, int dim, int hidden,
                            int n_heads, int n_kv_heads, int vocab, float rope_theta, float rms_eps,
                            int dtype, uint64_t seed, float std, int threads);
/* The same with the output head in its own type (the layers and tok_emb in dtype); both may
 * be JD_F32, JD_F16, JD_Q4_0, JD_Q5_0, JD_Q8_0, JD_Q4_K or JD_Q6_K (real host files often
 * carry a Q6_K head beside Q4_K layers). */
int jd_gguf_write_synthetic_mixed(const char *path, const char *arch, int n_layers, int dim, int hidden,
                                  int n_heads, int n_kv_heads, int vocab, float rope_theta, float rms_eps,
                                  int dtype, int out_dtype, uint64_t seed, float std, int threads);

/* ------------------------------------------------------------------------------------
 * GPU engine.
 * ---------------------------------------------------------------------------------- */
typedef struct jdg_ctx jdg_ctx;
typedef struct jdg_engine jdg_engine;

/* Per-step election trace, written for every (sequence, layer): k, elected slots in
 * election order, their softmax weights and the consensus EMA after the update.
 * Arrays are [B][n_layers] (k, ema) and [B][n_layers][16] (sel, w). */
typedef struct {
    int *k;
    int *sel;
    float *w;
    float *ema;
} jdg_trace;

int jdg_open(int device, jdg_ctx **out);
void jdg_close(jdg_ctx *ctx);
const char *jdg_last_error(jdg_ctx *ctx);
int jdg_device_count(int *n);

/* Upload an own model (alive experts, alive mask, per-layer consensus and temperature).
 * The host model stays the source of truth; max_batch sequence slots are allocated, each
 * with KV [n_layers][seq_len][kv_dim] f32 and its own consensus EMA per layer. */
int jdg_own_upload(jdg_ctx *ctx, const jd_model *m, int max_batch, jdg_engine **out);
/* Upload a host GGUF model: packed bytes copied as they are, LoRA parliament in f32.
 * KV holds max_seq positions per slot. */
int jdg_host_upload(jdg_ctx *ctx, const jd_host_model *h, int max_batch, int max_seq, jdg_engine **out);
/* Tensor-parallel host upload: this process holds rank `rank` of `world`; nccl_id is the
 * 128-byte ncclUniqueId created by rank 0 (jdg_comm_unique_id) and shared by the caller. */
int jdg_comm_unique_id(void *nccl_id_128);
int jdg_host_upload_tp(jdg_ctx *ctx, const jd_host_model *h, int max_batch, int max_seq, int rank, int world,
                       const void *nccl_id_128, jdg_engine **out);
void jdg_engine_free(jdg_engine *e);

/* Sampling: temperature <= 0 is greedy argmax (janusdoe.c:3637, 3374); otherwise
 * sample() with temperature and top_k and each sequence's own xorshift state. */
int jdg_set_sampling(jdg_engine *e, float temperature, int top_k);
/* Fresh sequence in slot `slot` (-1: all): zero its KV, restart its EMAs (chat(),
 * janusdoe.c:3656-3657), clear its prompt. */
int jdg_reset(jdg_engine *e, int slot);
/* Give slots 0..B-1 a prompt: tokens[b*P + i], i < len[b] <= P.  The next run feeds the
 * prompt token by token (sequential prefill, janusdoe.c:3660) and then generates. */
int jdg_set_prompt(jdg_engine *e, int B, const int *tokens, int P, const int *len, const uint64_t *rng);
/* Run n decode steps for slots 0..B-1 entirely on the device: each step forwards the
 * current token at the current position, then picks the next one (the prompt's while
 * it lasts, else sampled/greedy).  Generated tokens land in the history buffer. */
int jdg_run(jdg_engine *e, int B, int n_steps);
/* Hebbian --learn pass (host_learn_run, janusdoe.c:3416-3447) over the token stream toks on
 * the engine's LoRA parliament (one GPU): for t < nt-1 a forward of toks[t] at position t on
 * fresh caches of slot 0 (the EMA carries on), the prophecy-debt signal of toks[t+1], and a
 * notorch step (janusdoe.c:3102-3132) on every expert elected in that token, in layer and slot
 * order, then quarantine (janusdoe.c:3136-3144).  The reference's global RNG state and
 * notorch offset are explicit (in/out); *deaths receives the experts quarantined.  lr is the
 * reference's learning rate argument. */
int jdg_host_learn(jdg_engine *e, const int *toks, int nt, float lr, uint64_t *rng_state, int *notorch_offset,
                   int *deaths);
/* LoRA factors A [dim][rank], B [rank][dim] and alive flag of expert slot x of layer l as the
 * engine holds them (any pointer may be NULL). */
int jdg_host_get_expert(jdg_engine *e, int l, int x, float *A, float *B, int *alive);
/* Prompt prefill (own model; replaces the token-by-token prefill of chat(), janusdoe.c:3660):
 * right after jdg_set_prompt, runs every prompt token of slots 0..B-1 but the last through
 * the model as one batch per sequence and leaves each slot where len-1 jdg_run steps would:
 * KV cache and per-layer EMA filled, at position len-1 with the last prompt token next.
 * Elections use the EMA as an ordered scan over the tokens, so they equal token-by-token
 * decoding's.  JD_EUNSUPPORTED for a host-model engine (its prompts run through jdg_run). */
int jdg_prefill(jdg_engine *e, int B);
/* Election trace of the last prefilled sequence's first n prompt tokens ([n][n_layers]...). */
int jdg_get_prefill_trace(jdg_engine *e, int n, jdg_trace *trace);
/* Read back: current token and position per slot, and the last n history entries. */
int jdg_get_state(jdg_engine *e, int B, int *tok, int *pos);
int jdg_get_history(jdg_engine *e, int B, int n, int *tokens);
/* One decode step through host buffers: upload tok/pos (and rng if given), forward,
 * pick, download next_tok (and rng).  logits [B][vocab] and trace are optional. */
int jdg_step(jdg_engine *e, int B, const int *tok, const int *pos, uint64_t *rng, int *next_tok,
             float *logits, jdg_trace *trace);
/* Logits and trace of the last step for slots 0..B-1. */
int jdg_get_logits(jdg_engine *e, int B, float *logits);
int jdg_get_trace(jdg_engine *e, int B, jdg_trace *trace);
/* Timing: device time of the last jdg_run in milliseconds (CUDA events on the engine's stream). */
int jdg_last_run_ms(jdg_engine *e, float *ms);
/* Per-kernel device time of one more step (events around each launch of a step). */
int jdg_profile_step(jdg_engine *e, int B, float *ms_by_kernel, int max_kernels, int *n_kernels,
                     const char **names);
/* Device-side counters since the last jdg_reset_stats: [0] experts read (per step and
 * layer, the union over the batch of elected experts), [1] KV positions read (sum over
 * sequences of pos+1 per step), [2] decode steps. */
int jdg_get_stats(jdg_engine *e, uint64_t *out3);
int jdg_reset_stats(jdg_engine *e);
/* Debug timeline of the batch-1 kernel chain: the first call allocates it (later steps
 * record into it); out[slot*3+{0,1,2}] = earliest CTA entry, earliest return from the
 * dependency wait, latest CTA exit, in ns of the GPU global timer; each call re-arms it. */
int jdg_debug_timeline(jdg_engine *e, int n_slots, uint64_t *out);
/* Counts of this library's kernel launches since the engine was created. */
int jdg_launch_count(jdg_engine *e, long long *n);

/* Packed GEMV/GEMM on the device through host buffers: out[b][r] = W[r][:] . x[b][:],
 * W packed as dtype dt (JD_F32, JD_Q8_0, JD_Q4_K), B rows of x.  Mirrors jd_qmatvec
 * (janusdoe.c:2685): JD_EUNSUPPORTED where the reference returns -1. */
int jdg_qmatvec(jdg_ctx *ctx, float *out, const void *W, int dt, const float *x, int r, int c, int B);

/* No counterpart in the reference.  Greedy vocabulary pick for callers that cannot allocate
 * device memory (all their buffers come from another allocator or a preallocated pool):
 * logits_dev[r] = W_dev[r][:] . x_dev (W f32 row-major [rows][cols], cols a multiple of 4)
 * and *argmax_dev = the first index of the maximum, enqueued on `stream` (a cudaStream_t of
 * the current device, NULL for the default stream); returns once enqueued.  W_dev and x_dev
 * must be 16-byte aligned (rows and x are read as 16-byte vectors); logits_dev and argmax_dev
 * are written as scalars.  NaN logits are never picked; if no logit is greater than -inf the
 * pick is 0.  It calls no allocator: its scratch (per-CTA partial maxima and a completion
 * ticket) is a fixed device array of about 64 KB per GPU, held until the process exits,
 * which limits a call to 131072 rows and 16384 columns (larger sizes return JD_EINVAL,
 * message in jdg_last_error(NULL)).  The first call on a device looks up that array's
 * address, so make the first call before any stream capture.  All calls share the array:
 * calls that overlap on the GPU (other streams, other host threads) race and must be
 * serialised by the caller. */
int jdg_logits_argmax_noalloc(const float *W_dev, const float *x_dev, int rows, int cols, float *logits_dev,
                              int *argmax_dev, void *stream);
/* The argument check that jdg_logits_argmax_noalloc runs before it touches the GPU: null
 * pointers, shape, 16-byte alignment of W_dev and x_dev, and the scratch limits.  Pure host
 * arithmetic (no CUDA call, nothing dereferenced); JD_OK or JD_EINVAL with the message in
 * jdg_last_error(NULL). */
int jdg_logits_argmax_noalloc_check(const void *W_dev, const void *x_dev, int rows, int cols, const void *logits_dev,
                                    const void *argmax_dev);
#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif

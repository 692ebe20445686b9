/*
 * m_cli.c — the `m` command line, the token-loop surface of the reference's main()
 * (janusdoe.c:3734-3811) on the B200 engine:
 *
 *   m --depth N [--gguf m.gguf] [--seed S] [--vocab V] [--ask TEXT] [--gen N]
 *               [--temp T] [--topk K]
 *       own model: weights from the GGUF the reference exports (load_own_gguf semantics),
 *       or seeded synthetic weights; the prompt's bytes are the reference's byte tokens
 *       (ids 0..255, janusdoe.c:228); chat() samples at temperature 0.8, top-k 40.
 *   m --host model.gguf [--ask TEXT] [--rope-neox | --rope-norm] [--lora FILE]
 *               [--lora-rank R] [--gen N] [--learn FILE]
 *       host mode (janusdoe.c:3762-3795): gguf_host_load, BOS + whole-word tokenisation
 *       (jd_host_tokenize), greedy generation with the LoRA parliament, stop at EOS.
 *   --print-ids prints the prompt's and the generated token ids after the text.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "jdgpu.h"

static void usage(void) {
    printf("m — Democracy of Experts token loop on B200.\n\n");
    printf("  --depth N       own model depth (dim = 64*N, clamped to [128, 768])\n");
    printf("  --gguf PATH     own-model weights exported by the trainer (m.gguf)\n");
    printf("  --seed S        seeded synthetic weights when no GGUF is given (default 0)\n");
    printf("  --vocab V       vocabulary size (default 258 + BPE merges for the depth)\n");
    printf("  --host GGUF     index a llama-family model and generate through it\n");
    printf("  --ask \"PROMPT\"  prompt (default: a sample)\n");
    printf("  --rope-neox     force NeoX RoPE pairing; --rope-norm forces NORM pairing\n");
    printf("  --lora FILE     LoRA parliament sidecar for --host (default: drawn from --seed)\n");
    printf("  --gen N         tokens to generate (default 64)\n");
    printf("  --temp T --topk K   own-model sampling (default 0.8 and 40, as chat())\n");
    printf("  --learn FILE    --host: Hebbian LoRA pass over the file's tokens (lr 0.01) before generating\n");
    printf("  --print-ids     also print the prompt and generated token ids\n");
}

/* the whole file as a NUL-terminated string (NULL on failure) */
static char *read_text(const char *path) {
    FILE *f = fopen(path, "rb");
    if (!f) return NULL;
    fseek(f, 0, SEEK_END);
    long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    char *t = n >= 0 ? malloc((size_t)n + 1) : NULL;
    if (t && fread(t, 1, (size_t)n, f) != (size_t)n) { free(t); t = NULL; }
    if (t) t[n] = 0;
    fclose(f);
    return t;
}

static void print_ids(const char *what, const int *ids, int n) {
    printf("[ids] %s", what);
    for (int i = 0; i < n; i++) printf(" %d", ids[i]);
    printf("\n");
}

static int fail(jdg_ctx *ctx, const char *what, int rc) {
    fprintf(stderr, "[m] %s failed (%d): %s\n", what, rc, jdg_last_error(ctx));
    return 1;
}

int main(int argc, char **argv) {
    int depth = 0, gen = 64, topk = 40, rope_override = -1, vocab = 0, lora_rank = 16, show_ids = 0;
    uint64_t seed = 0;
    float temp = 0.8f;
    const char *gguf = NULL, *host = NULL, *ask = "The capital of France is", *lora = NULL, *learn = NULL;
    for (int i = 1; i < argc; i++) {
        if (!strcmp(argv[i], "--depth") && i + 1 < argc) depth = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--gguf") && i + 1 < argc) gguf = argv[++i];
        else if (!strcmp(argv[i], "--seed") && i + 1 < argc) seed = strtoull(argv[++i], NULL, 10);
        else if (!strcmp(argv[i], "--vocab") && i + 1 < argc) vocab = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--host") && i + 1 < argc) host = argv[++i];
        else if (!strcmp(argv[i], "--ask") && i + 1 < argc) ask = argv[++i];
        else if (!strcmp(argv[i], "--lora") && i + 1 < argc) lora = argv[++i];
        else if (!strcmp(argv[i], "--learn") && i + 1 < argc) learn = argv[++i];
        else if (!strcmp(argv[i], "--lora-rank") && i + 1 < argc) lora_rank = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--gen") && i + 1 < argc) gen = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--temp") && i + 1 < argc) temp = (float)atof(argv[++i]);
        else if (!strcmp(argv[i], "--topk") && i + 1 < argc) topk = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--rope-neox")) rope_override = 0;
        else if (!strcmp(argv[i], "--rope-norm")) rope_override = 1;
        else if (!strcmp(argv[i], "--print-ids")) show_ids = 1;
        else if (!strcmp(argv[i], "--help") || !strcmp(argv[i], "-h")) { usage(); return 0; }
    }
    if (!host && depth <= 0) { usage(); return 1; }
    if (gen < 1) gen = 1;
    jdg_ctx *ctx = NULL;
    int rc = jdg_open(0, &ctx);
    if (rc != JD_OK) return fail(NULL, "jdg_open", rc);
    jdg_engine *eng = NULL;
    if (host) {
        jd_host_model hm;
        if ((rc = jd_host_load_gguf(&hm, host, rope_override, lora_rank)) != JD_OK) return fail(ctx, "loading the host GGUF", rc);
        rc = lora ? jd_host_lora_load(&hm, lora) : jd_host_lora_seed(&hm, seed, 4, 0.02f / 4.0f, 0.02f);
        if (rc != JD_OK) return fail(ctx, "LoRA parliament", rc);
        printf("[m] host %s: arch=%s rope=%s dim=%d layers=%d heads=%d/%d vocab=%d\n", host, hm.arch,
               hm.rope_norm ? "NORM" : "NEOX", hm.dim, hm.n_layers, hm.n_heads, hm.n_kv_heads, hm.vocab);
        const int max_seq = 512;
        int toks[256], nt = 0;
        if (hm.bos >= 0 && hm.bos < hm.vocab) toks[nt++] = hm.bos;
        if (hm.vocab_tokens) nt += jd_host_tokenize(&hm, ask, toks + nt, 200);
        if (nt == 0) toks[nt++] = 1;
        if (gen > max_seq - nt) gen = max_seq - nt;
        if ((rc = jdg_host_upload(ctx, &hm, 1, max_seq, &eng)) != JD_OK) return fail(ctx, "upload", rc);
        if (learn) {  /* janusdoe.c:3776-3788: tokens of the file (at most 512), one learning pass */
            char *text = read_text(learn);
            if (text && hm.vocab_tokens) {
                int lt[512], nl = jd_host_tokenize(&hm, text, lt, 512), deaths = 0, offset = 0;
                uint64_t rng = 42; /* the reference's RNG state after loading */
                if ((rc = jdg_host_learn(eng, lt, nl, 0.01f, &rng, &offset, &deaths)) != JD_OK)
                    return fail(ctx, "learn", rc);
                printf("[learn] %s: %d tokens | quarantined %d\n", learn, nl, deaths);
            } else {
                printf("[learn] cannot read %s or host has no vocab\n", learn);
            }
            free(text);  /* the EMA carries into the generation, as in the reference */
        }
        if ((rc = jdg_set_prompt(eng, 1, toks, nt, &nt, NULL)) != JD_OK) return fail(ctx, "prompt", rc);
        if ((rc = jdg_run(eng, 1, nt - 1 + gen)) != JD_OK) return fail(ctx, "decode", rc);
        int *out = malloc(sizeof(int) * gen);
        jdg_get_history(eng, 1, gen, out);
        float ms = 0;
        jdg_last_run_ms(eng, &ms);
        printf("[host] %s", ask);
        int ng = 0;
        for (; ng < gen; ng++) {
            if (hm.eos >= 0 && out[ng] == hm.eos) break;
            char tb[512];
            if (hm.vocab_tokens && jd_host_token_text(&hm, out[ng], tb, sizeof tb) >= 0) fputs(tb, stdout);
            else printf(" %d", out[ng]);
        }
        printf("\n[m] %d steps in %.2f ms on the GPU\n", nt - 1 + gen, ms);
        if (show_ids) {
            print_ids("prompt", toks, nt);
            print_ids("generated", out, ng);
        }
        free(out);
        jdg_engine_free(eng);
        jd_host_free(&hm);
    } else {
        jd_config c;
        jd_config_from_depth(depth, &c);
        if (vocab > 0) c.vocab_size = vocab;
        jd_model m;
        if ((rc = jd_model_alloc(&m, &c)) != JD_OK) return fail(ctx, "model alloc", rc);
        if (gguf) rc = jd_model_load_gguf(&m, gguf);
        else rc = jd_model_fill_seeded(&m, seed, 0.02f, 0);
        if (rc != JD_OK) return fail(ctx, gguf ? "loading the model GGUF" : "seeding", rc);
        printf("[m] depth %d: dim=%d heads=%d/%d experts=%d hidden=%d vocab=%d\n", c.depth, c.dim, c.n_heads,
               c.n_kv_heads, c.initial_experts, c.hidden_dim, c.vocab_size);
        int n = (int)strlen(ask);
        if (n > c.seq_len - 1) n = c.seq_len - 1;
        if (n < 1) n = 1;
        int *ids = malloc(sizeof(int) * n);
        for (int i = 0; i < n; i++) ids[i] = (unsigned char)ask[i];
        if (gen > c.seq_len - n) gen = c.seq_len - n;
        uint64_t rng = 42;
        if ((rc = jdg_own_upload(ctx, &m, 1, &eng)) != JD_OK) return fail(ctx, "upload", rc);
        jdg_set_sampling(eng, temp, topk);
        if ((rc = jdg_set_prompt(eng, 1, ids, n, &n, &rng)) != JD_OK) return fail(ctx, "prompt", rc);
        if ((rc = jdg_run(eng, 1, n - 1 + gen)) != JD_OK) return fail(ctx, "decode", rc);
        int *out = malloc(sizeof(int) * gen);
        jdg_get_history(eng, 1, gen, out);
        float ms = 0;
        jdg_last_run_ms(eng, &ms);
        printf("> %s\n  ", ask);
        for (int i = 0; i < gen; i++) {
            if (out[i] == 257) break; /* <EOS> (janusdoe.c:228) */
            if (out[i] < 256) putchar(out[i] >= 32 && out[i] < 127 ? out[i] : '.');
            else printf("<%d>", out[i]);
        }
        printf("\n[m] %d steps in %.2f ms on the GPU\n", n - 1 + gen, ms);
        if (show_ids) {
            int ng = 0;
            while (ng < gen && out[ng] != 257) ng++;
            print_ids("prompt", ids, n);
            print_ids("generated", out, ng);
        }
        free(out);
        free(ids);
        jdg_engine_free(eng);
        jd_model_free(&m);
    }
    jdg_close(ctx);
    return 0;
}

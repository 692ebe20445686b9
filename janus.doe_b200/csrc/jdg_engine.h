// jdg_engine.h — engine state shared by the own-model and host-model halves of the library.
#pragma once
#include <cuda_runtime.h>

#include <map>
#include <vector>

#include "../../include/jdgpu.h"
#include "jdg_common.cuh"

struct LayerDev {
    float *attn_norm = nullptr, *ffn_norm = nullptr, *wqkv = nullptr, *wo = nullptr, *w_vote = nullptr;
    float temperature = 0.f;
    // tensor-core blocks (TF32 hi/lo, jdg_tc32.cuh) of q/k/v and Wo; per expert slot the
    // gate/up and down blocks, as device tables of 16 pointers (null for dead slots)
    uint8_t *tc_wqkv = nullptr, *tc_wo = nullptr;
    const uint8_t **tc_gu = nullptr, **tc_dn = nullptr;
    const uint8_t **tc_wqkv_tab = nullptr, **tc_wo_tab = nullptr;  // one-entry tables
};

// packed host-model weight on the device (layout chosen by jdg_host.cu at upload)
struct PackedW {
    int dt = 0;              // JD_F32, JD_Q8_0, JD_Q4_K
    int rows = 0, cols = 0;
    const void *q = nullptr;  // quant codes (or f32 values)
    const void *s = nullptr;  // per-block scales / headers
};

struct HostLayerDev {
    PackedW wqkv, wo, gu, down;  // fused q|k|v rows; gate/up interleaved per row tile
    float *attn_norm = nullptr, *ffn_norm = nullptr;  // null = ones
    float *w_vote = nullptr;                          // [16][D]
    int *alive = nullptr;                             // [16] device
    float *lora_A = nullptr, *lora_B = nullptr;       // [16][D][R], [16][R][D] (dead slots zero)
    float focus = 1.f, attn_bias = 0.f;
};

struct jdg_engine {
    jdg_ctx *ctx = nullptr;
    int kind = 0;  // 0 own model, 1 host GGUF model
    cudaStream_t st = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    std::vector<void *> allocs;
    // shapes
    int B_max = 0, L = 0, D = 0, Hh = 0, KVH = 0, HD = 0, hidden = 0, V = 0, max_seq = 0;
    int qd = 0, kd = 0, qkvd = 0, nchunk = 0, kmax = 1;
    int attn_rows = 0;                   // 1: k_attn_rows (32-position chunks), 0: k_attn_partial
    int ldl = 0;  // logits row stride (the rank's vocab slice under tensor parallelism)
    float eps = 1e-5f, clamp = 0.f;
    int rope_norm = 0;
    int n_alive[JD_MAX_LAYERS] = {0};
    float layer_consensus[JD_MAX_LAYERS] = {0};
    // own-model weights
    void *arena = nullptr;
    float *tok_emb = nullptr, *output = nullptr, *output_norm = nullptr;
    LayerDev layers[JD_MAX_LAYERS];
    float **gu_tab = nullptr, **dn_tab = nullptr;
    int *alive_dev = nullptr;
    float *rope_cos = nullptr, *rope_sin = nullptr;
    // host-model weights
    HostLayerDev hl[JD_MAX_LAYERS];
    PackedW out_w;
    int lora_rank = 0;
    float lora_alpha = 0.1f;
    void *host_priv = nullptr;  // jdg_host.cu state (NCCL communicator, TP shard info)
    // activations
    float *x = nullptr, *xb = nullptr, *qkv = nullptr, *att = nullptr, *part = nullptr, *hbuf = nullptr, *ybuf = nullptr;
    float *logits = nullptr, *xn = nullptr, *lora_t = nullptr;
    int *kcnt = nullptr, *sel = nullptr;
    float *selw = nullptr;
    int *rcnt = nullptr, *ridx = nullptr, *pairrow = nullptr;
    // per-sequence state
    int *tok = nullptr, *pos = nullptr, *plen = nullptr, *prompt = nullptr, *hist = nullptr, *hist_n = nullptr,
        *next_out = nullptr;
    uint64_t *rng = nullptr;
    float *consensus = nullptr;
    int Pmax = 0, Hmax = 0;
    float *kc = nullptr, *vc = nullptr;
    long kv_bstride = 0;
    int *err = nullptr;
    unsigned *tickets = nullptr;  // last-CTA counters of the batch-1 chain (1024)
    float *amax_v = nullptr, *vpart = nullptr, *ffn_inv = nullptr;
    const float **sel_gu = nullptr, **sel_dn = nullptr;
    float *ema_new = nullptr, *x2 = nullptr;  // x2: ping-pong residual of the batch-1 chain  // elected expert weights (batch-1 chain)
    unsigned long long *stats = nullptr;
    unsigned long long *timeline = nullptr;  // optional per-kernel timeline (jdg_debug_timeline)  // [0] experts read, [1] KV positions read, [2] steps
    int *pin_tok = nullptr, *pin_pos = nullptr, *pin_next = nullptr;  // pinned staging for jdg_step
    int *pin_err = nullptr;              // pinned copy of the device error word
    int *amax_i = nullptr;
    int b1_ok = 0;                // shapes fit the batch-1 PDL chain
    int force_generic = 0;        // JDG_GENERIC=1: use the generic kernels at batch 1
    int force_chain = 1;          // batch 1: the kernel chain (JDG_B1=step selects the persistent step)
    void *b1p_layers = nullptr;   // per-layer table of the persistent batch-1 step (B1PLayer[L])
    int b1p_grid = 0;             // CTAs of the persistent step (0: not usable)
    int *tr_k = nullptr, *tr_sel = nullptr;
    float *tr_w = nullptr, *tr_ema = nullptr;
    // tensor-core GEMMs of the batched own-model step (jdg_tc32.cuh)
    int tc_ok = 0;                       // blocks built; JDG_SIMT_GEMM=1 keeps the SIMT kernels
    uint8_t *tc_out = nullptr;           // LM head blocks
    const uint8_t **tc_out_tab = nullptr;
    uint8_t *tc_xt = nullptr;            // activation blocks, sized for 16 segments
    size_t tc_xt_bytes = 0;
    float *tc_part = nullptr;            // split-K partials
    // prompt prefill buffers (own model, allocated at the first jdg_prefill; rows = tokens)
    float *pf_x = nullptr, *pf_xb = nullptr, *pf_qkv = nullptr, *pf_att = nullptr, *pf_part = nullptr;
    float *pf_hbuf = nullptr, *pf_ybuf = nullptr, *pf_selw = nullptr, *pf_votes = nullptr, *pf_cs = nullptr;
    int *pf_kcnt = nullptr, *pf_sel = nullptr, *pf_rcnt = nullptr, *pf_ridx = nullptr, *pf_pairrow = nullptr;
    int *pf_pos = nullptr, *pf_tr_k = nullptr, *pf_tr_sel = nullptr;
    float *pf_tr_w = nullptr, *pf_tr_ema = nullptr;
    int pf_last_n = 0;                 // tokens of the last prefill (its trace rows)
    std::vector<int> prompt_host, plen_host;  // copies of the last jdg_set_prompt
    // sampling
    float temp = 0.f;
    int top_k = 0;
    // graphs and counters
    std::map<int, cudaGraphExec_t> graphs;
    std::map<int, long long> launches_per_step;
    long long launches = 0;
    float last_ms = 0.f;
};

void jdg_set_err(jdg_ctx *c, const char *fmt, ...);
int jdg_ctx_device(jdg_ctx *c);
int jdg_alloc_state(jdg_engine *e);
int jdg_own_upload_impl(jdg_engine *e, const jd_model *m, int max_batch);
void jdg_launch_rope(jdg_engine *e, int l, int B, SplitPart sp = SplitPart{nullptr, 1, 1});
void jdg_launch_attention(jdg_engine *e, int l, int B, float scale, float bias);
int jdg_attn_setup(jdg_engine *e);
void jdg_launch_pick(jdg_engine *e, int B);
void jdg_launch_pick_tp(jdg_engine *e, int B, const float *v, const int *ix, int world);
int jdg_engine_create(jdg_ctx *ctx, int kind, jdg_engine **out);
void jdg_launch_elect(jdg_engine *e, int l, int B, const float *xin, const float *norm_w, const float *w_vote,
                      const int *alive, float temperature, int host, SplitPart sp = SplitPart{nullptr, 1, 1});
// host-model half (jdg_host.cu)
int jdg_enqueue_host_step(jdg_engine *e, int B);
int jdg_host_set_attrs(jdg_engine *e);
void jdg_host_release(jdg_engine *e);

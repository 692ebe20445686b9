// jdg_host.cu — host GGUF model half of the engine: upload (repacking packed Q8_0/Q4_K
// rows losslessly, tensor-parallel sharding), the decode step (gguf_host_forward,
// janusdoe.c:3160-3322, for a batch of independent sequences), NCCL all-reduce for the
// tensor-parallel case, and the standalone packed GEMV entry point.
#include <cudaTypedefs.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

#include "jdg_engine.h"
#include "jdg_hb1.cuh"
#include "jdg_hpar.cuh"
#include "jdg_learn.cuh"
#include "jdg_qmma.cuh"

using namespace jdg;

#define E_CTX (e->ctx)
#define CK(call)                                                                                                    \
    do {                                                                                                            \
        cudaError_t _e = (call);                                                                                    \
        if (_e != cudaSuccess) {                                                                                    \
            jdg_set_err(E_CTX, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(_e), __FILE__, __LINE__);         \
            return JD_ECUDA;                                                                                        \
        }                                                                                                           \
    } while (0)
#define NK(call)                                                                                                    \
    do {                                                                                                            \
        ncclResult_t _r = (call);                                                                                   \
        if (_r != ncclSuccess) {                                                                                    \
            jdg_set_err(E_CTX, "%s failed: %s", #call, ncclGetErrorString(_r));                                     \
            return JD_ECOMM;                                                                                        \
        }                                                                                                           \
    } while (0)

namespace {

struct HostPriv {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    int H_loc = 0, KVH_loc = 0, hidden_loc = 0, V_loc = 0, V_off = 0;
    float *partial = nullptr;               // [B][D] partial sums to all-reduce
    float *amx_v = nullptr;                 // [world][B]
    int *amx_i = nullptr;
    float *amx_v_loc = nullptr;
    int *amx_i_loc = nullptr;
    float *lora_A[JD_MAX_LAYERS] = {}, *lora_B[JD_MAX_LAYERS] = {};
    QW wqkv[JD_MAX_LAYERS], wo[JD_MAX_LAYERS], gu[JD_MAX_LAYERS], dn[JD_MAX_LAYERS];
    QW out;
    float *ones = nullptr;                  // [D] of 1.0f for absent norms
    // batch-1 chain (jdg_hb1.cuh)
    bool hb1 = false;                       // shapes and dtypes fit the chain
    int *alive_list[JD_MAX_LAYERS] = {};    // alive expert ids, ascending
    int gu_ctas = 0, lm_ctas = 0;           // persistent grids: resident CTAs on all SMs
    int n_sm = 148;
    float *votes = nullptr, *tall = nullptr;
    uint8_t *xprep = nullptr;               // batched Q4_K GEMM: activations as fp16 hi/lo tiles
    float *qm_part = nullptr;               // split-K partials
    unsigned *qm_tickets = nullptr;         // split-K row-tile tickets
    std::vector<QmMaps> qm_maps;            // TMA tensor maps of the Q4_K matrices the GEMM reads
    // batched LoRA parliament (jdg_hpar.cuh)
    float *hpar_part = nullptr;             // [D/256][16][R+1][32] partial dots
    unsigned *hpar_tickets = nullptr;       // [17]
    float *hpar_votes = nullptr;            // [max_batch][16]
    float *hpar_tall = nullptr;             // [max_batch][16][R]
    // the votes/projections/elections of a layer run on a second stream, forked after the
    // q/k/v GEMM (they read only the normed layer input) and joined before the LoRA apply
    cudaStream_t st2 = nullptr;
    std::vector<cudaEvent_t> ev_fork, ev_join;  // one pair per layer
    // Hebbian --learn (jdg_learn.cuh): captures of the forward, signal, update list
    bool learn_on = false;                  // the generic step captures dy and x
    float *learn_dyraw = nullptr, *learn_x = nullptr, *learn_dy = nullptr, *learn_sig = nullptr;
    int *learn_next = nullptr, *learn_dead = nullptr;
    LearnUpd *learn_upd = nullptr;
    float **learn_A = nullptr, **learn_B = nullptr;
    int **learn_alive = nullptr;
};

HostPriv *priv(jdg_engine *e) { return (HostPriv *)e->host_priv; }

// cuTensorMapEncodeTiled from the driver (through the runtime, no link-time dependency)
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// The two tensor maps k_qm_q4k reads a Q4_K matrix through: the code bytes [rows][cols/2]
// in boxes of 128 bytes x 128 rows with the 128-byte swizzle, and the 16-byte superblock
// headers [rows][cols/256 * 16] in boxes of 16 bytes x 128 rows.  Created once per matrix.
int qm_add_maps(jdg_engine *e, const QW &w) {
    HostPriv *hp = priv(e);
    for (const QmMaps &m : hp->qm_maps)
        if (m.q == w.q) return JD_OK;
    auto enc = tensor_map_encoder();
    if (!enc) {
        jdg_set_err(e->ctx, "cuTensorMapEncodeTiled is not available from the driver");
        return JD_ECUDA;
    }
    QmMaps m;
    m.q = w.q;
    const cuuint32_t es[2] = {1, 1};
    const cuuint64_t gd[2] = {(cuuint64_t)w.cols / 2, (cuuint64_t)w.rows}, gs[1] = {(cuuint64_t)w.cols / 2};
    const cuuint32_t box[2] = {128, 128};
    CUresult r = enc(&m.codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(w.q), gd, gs, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    const cuuint64_t hd[2] = {(cuuint64_t)(w.cols / 256) * 16, (cuuint64_t)w.rows}, hs[1] = {(cuuint64_t)(w.cols / 256) * 16};
    const cuuint32_t hbox[2] = {16, 128};
    if (r == CUDA_SUCCESS)
        r = enc(&m.hdr, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(w.s), hd, hs, hbox, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        jdg_set_err(e->ctx, "cuTensorMapEncodeTiled failed (%d) for a %d x %d Q4_K matrix", (int)r, w.rows, w.cols);
        return JD_ECUDA;
    }
    hp->qm_maps.push_back(m);
    return JD_OK;
}
const QmMaps *qm_find_maps(jdg_engine *e, const QW &w) {
    for (const QmMaps &m : priv(e)->qm_maps)
        if (m.q == w.q) return &m;
    return nullptr;
}

// source block geometry of the GGUF types the upload accepts packed
int block_elems(int dt) {
    switch (dt) {
    case JD_F32: case JD_F16: return 1;
    case JD_Q4_0: case JD_Q5_0: case JD_Q8_0: return 32;
    case JD_Q4_K: case JD_Q6_K: return 256;
    default: return 0;
    }
}
size_t block_bytes(int dt) {
    switch (dt) {
    case JD_F32: return 4;
    case JD_F16: return 2;
    case JD_Q4_0: return 18;
    case JD_Q5_0: return 22;
    case JD_Q8_0: return 34;
    case JD_Q4_K: return 144;
    case JD_Q6_K: return 210;
    default: return 0;
    }
}

// register bucket of the batch-1 chain for a packed matrix (0: not supported there)
int hb1_maxc(const QW &w) {
    if (w.dt != JD_Q8_0 && w.dt != JD_Q4_K) return 0;
    const int n = prow_chunks(w.dt, w.cols);
    return n <= 4 ? 4 : n <= 8 ? 8 : n <= 12 ? 12 : n <= 16 ? 16 : 0;
}

// Host-side repack of selected rows (and a block-aligned column range) of a packed tensor
// into the device layout described in jdg_host_kernels.cuh.
struct Packed {
    std::vector<uint8_t> q, s;
    int dt = 0, rows = 0, cols = 0;
};
bool repack(const void *src, int dt, int src_cols, const std::vector<int> &rows, int c0, int c1, Packed &out) {
    const int be = block_elems(dt);
    if (!be || src_cols % be || c0 % be || c1 % be || c1 <= c0) return false;
    const size_t bb = block_bytes(dt), row_bytes = (size_t)(src_cols / be) * bb;
    const int nb = (c1 - c0) / be, cols = c1 - c0;
    out.dt = dt;
    out.rows = (int)rows.size();
    out.cols = cols;
    const uint8_t *base = (const uint8_t *)src;
    if (dt == JD_F32) {
        out.q.resize((size_t)out.rows * cols * 4);
        for (size_t r = 0; r < rows.size(); r++)
            memcpy(&out.q[r * cols * 4], base + (size_t)rows[r] * row_bytes + (size_t)c0 * 4, (size_t)cols * 4);
    } else if (dt == JD_F16) {
        // half -> float is exact: stored as f32 rows
        out.dt = JD_F32;
        out.q.resize((size_t)out.rows * cols * 4);
        for (size_t r = 0; r < rows.size(); r++) {
            const uint8_t *rp = base + (size_t)rows[r] * row_bytes + (size_t)c0 * 2;
            float *o = reinterpret_cast<float *>(&out.q[r * cols * 4]);
            for (int j = 0; j < cols; j++) o[j] = jdq_half_at(rp + 2 * j);
        }
    } else if (dt == JD_Q4_0 || dt == JD_Q5_0) {
        // 4/5-bit codes with one f16 scale per 32 weights: the value (q - 8)*d or (q - 16)*d is
        // an int8 code times the same scale, so they are stored in the Q8_0 layout exactly
        const int bias = dt == JD_Q4_0 ? 8 : 16;
        out.dt = JD_Q8_0;
        out.q.resize((size_t)out.rows * cols);
        out.s.resize((size_t)out.rows * nb * 2);
        for (size_t r = 0; r < rows.size(); r++) {
            const uint8_t *rp = base + (size_t)rows[r] * row_bytes + (size_t)(c0 / 32) * bb;
            for (int b = 0; b < nb; b++) {
                const uint8_t *blk = rp + (size_t)b * bb, *nib = blk + (dt == JD_Q4_0 ? 2 : 6);
                const uint32_t fifth = dt == JD_Q5_0 ? (uint32_t)blk[2] | ((uint32_t)blk[3] << 8) |
                                                           ((uint32_t)blk[4] << 16) | ((uint32_t)blk[5] << 24)
                                                     : 0u;
                memcpy(&out.s[(r * nb + b) * 2], blk, 2);
                int8_t *codes = reinterpret_cast<int8_t *>(&out.q[r * cols + (size_t)b * 32]);
                for (int w = 0; w < 32; w++) {
                    const int q = ((w < 16 ? nib[w] : nib[w - 16] >> 4) & 15) | (int)(((fifth >> w) & 1u) << 4);
                    codes[w] = (int8_t)(q - bias);
                }
            }
        }
    } else if (dt == JD_Q6_K) {
        // low-nibble bytes of every superblock [rows][K/2], then the 2-bit high parts
        // [rows][K/4], both in file order; headers [rows][K/256][32]: 16 int8 scales, f16 d
        out.q.resize((size_t)out.rows * cols / 2 + (size_t)out.rows * cols / 4);
        out.s.assign((size_t)out.rows * nb * 32, 0);
        uint8_t *ql = out.q.data(), *qh = out.q.data() + (size_t)out.rows * cols / 2;
        for (size_t r = 0; r < rows.size(); r++) {
            const uint8_t *rp = base + (size_t)rows[r] * row_bytes + (size_t)(c0 / 256) * 210;
            for (int b = 0; b < nb; b++) {
                const uint8_t *blk = rp + (size_t)b * 210;
                memcpy(ql + r * (cols / 2) + (size_t)b * 128, blk, 128);
                memcpy(qh + r * (cols / 4) + (size_t)b * 64, blk + 128, 64);
                memcpy(&out.s[(r * nb + b) * 32], blk + 192, 18);
            }
        }
    } else if (dt == JD_Q8_0) {
        out.q.resize((size_t)out.rows * cols);
        out.s.resize((size_t)out.rows * nb * 2);
        for (size_t r = 0; r < rows.size(); r++) {
            const uint8_t *rp = base + (size_t)rows[r] * row_bytes + (size_t)(c0 / 32) * 34;
            for (int b = 0; b < nb; b++) {
                memcpy(&out.s[(r * nb + b) * 2], rp + (size_t)b * 34, 2);
                memcpy(&out.q[r * cols + (size_t)b * 32], rp + (size_t)b * 34 + 2, 32);
            }
        }
    } else if (dt == JD_Q4_K) {
        out.q.resize((size_t)out.rows * cols / 2);
        out.s.resize((size_t)out.rows * nb * 16);
        for (size_t r = 0; r < rows.size(); r++) {
            const uint8_t *rp = base + (size_t)rows[r] * row_bytes + (size_t)(c0 / 256) * 144;
            for (int b = 0; b < nb; b++) {
                memcpy(&out.s[(r * nb + b) * 16], rp + (size_t)b * 144, 16);
                memcpy(&out.q[r * (cols / 2) + (size_t)b * 128], rp + (size_t)b * 144 + 16, 128);
            }
        }
    } else {
        return false;
    }
    return true;
}

std::vector<int> range(int a, int b) {
    std::vector<int> v;
    for (int i = a; i < b; i++) v.push_back(i);
    return v;
}

}  // namespace

static int dalloc(jdg_engine *e, void **p, size_t bytes) {
    cudaError_t r = cudaMalloc(p, bytes ? bytes : 256);
    if (r != cudaSuccess) {
        jdg_set_err(e->ctx, "cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(r));
        return JD_ENOMEM;
    }
    e->allocs.push_back(*p);
    return JD_OK;
}
#define DALLOC(ptr, bytes)                                       \
    do {                                                         \
        int _r = dalloc(e, (void **)&(ptr), (size_t)(bytes));    \
        if (_r != JD_OK) return _r;                              \
    } while (0)

static int upload_packed(jdg_engine *e, const Packed &p, QW &w) {
    w.dt = p.dt;
    w.rows = p.rows;
    w.cols = p.cols;
    uint8_t *q = nullptr, *s = nullptr;
    DALLOC(q, p.q.size());
    CK(cudaMemcpy(q, p.q.data(), p.q.size(), cudaMemcpyHostToDevice));
    if (!p.s.empty()) {
        DALLOC(s, p.s.size());
        CK(cudaMemcpy(s, p.s.data(), p.s.size(), cudaMemcpyHostToDevice));
    }
    w.q = q;
    w.s = s;
    return JD_OK;
}

static int upload_f32(jdg_engine *e, const float *src, size_t n, float **dst) {
    DALLOC(*dst, n * 4);
    CK(cudaMemcpy(*dst, src, n * 4, cudaMemcpyHostToDevice));
    return JD_OK;
}

int jdg_alloc_state(jdg_engine *e);
int jdg_reset(jdg_engine *e, int slot);
int jdg_host_set_attrs(jdg_engine *e);

// resident 128-thread CTAs per SM of the chain's GU (which 0) or LM (which 1) kernel for w
static int hb1_resident(const QW &w, size_t smem, int which) {
    int nb = 0;
#define OCC(DTV, MC)                                                                                            \
    (which ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k_hb1_lm<DTV, MC>, 128, smem)                    \
           : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k_hb1_gu<DTV, MC>, 128, smem))
    switch (w.dt * 100 + hb1_maxc(w)) {
    case 804: OCC(8, 4); break;
    case 808: OCC(8, 8); break;
    case 812: OCC(8, 12); break;
    case 816: OCC(8, 16); break;
    case 1204: OCC(12, 4); break;
    case 1208: OCC(12, 8); break;
    case 1212: OCC(12, 12); break;
    default: OCC(12, 16); break;
    }
#undef OCC
    return nb;
}

static int host_upload_impl(jdg_engine *e, const jd_host_model *h, int max_batch, int max_seq, int rank, int world) {
    HostPriv *hp = priv(e);
    const int D = h->dim, Hh = h->n_heads, KVH = h->n_kv_heads, HD = h->head_dim, HH = h->hidden;
    const int L = std::min(h->n_layers, JD_MAX_LAYERS);
    jd_tp_shard sh;
    if (jd_tp_shard_of(h, rank, world, &sh) != JD_OK) {
        jdg_set_err(e->ctx, "heads %d/%d or hidden %d not divisible by %d ranks", Hh, KVH, HH, world);
        return JD_EINVAL;
    }
    hp->rank = rank;
    hp->world = world;
    hp->H_loc = sh.q_heads;
    hp->KVH_loc = sh.kv_heads;
    hp->hidden_loc = sh.hidden;
    hp->V_off = sh.vocab0;
    hp->V_loc = sh.vocab;
    e->B_max = max_batch;
    e->L = L;
    e->D = D;
    e->Hh = hp->H_loc;
    e->KVH = hp->KVH_loc;
    e->HD = HD;
    e->hidden = hp->hidden_loc;
    e->V = h->vocab;
    e->ldl = std::max(1, hp->V_loc);
    e->max_seq = max_seq;
    e->qd = hp->H_loc * HD;
    e->kd = hp->KVH_loc * HD;
    e->qkvd = e->qd + 2 * e->kd;
    e->eps = h->rms_eps;
    e->clamp = 0.f;
    e->rope_norm = h->rope_norm;
    if (jdg_attn_setup(e) != JD_OK) return JD_ECUDA;
    e->lora_rank = h->lora_rank;
    e->lora_alpha = h->lora_alpha;
    const int R = h->lora_rank;
    // --- weights
    for (int l = 0; l < L; l++) {
        const jd_host_layer &ly = h->layers[l];
        if (!ly.wq || !ly.wk || !ly.wv || !ly.wo || !ly.gate || !ly.up || !ly.down) {
            jdg_set_err(e->ctx, "layer %d lacks attention or FFN weights", l);
            return JD_EUNSUPPORTED;
        }
        if (ly.wq_dt != ly.wk_dt || ly.wq_dt != ly.wv_dt || ly.gate_dt != ly.up_dt) {
            jdg_set_err(e->ctx, "layer %d mixes dtypes inside q/k/v or gate/up", l);
            return JD_EUNSUPPORTED;
        }
        // q|k|v rows of this rank's heads
        Packed pq, pk, pv, po, pg, pu, pd, pqkv, pgu;
        const int q0 = sh.q_head0 * HD, q1 = q0 + sh.q_heads * HD;
        const int k0 = sh.kv_head0 * HD, k1 = k0 + sh.kv_heads * HD;
        if (!repack(ly.wq, ly.wq_dt, D, range(q0, q1), 0, D, pq) || !repack(ly.wk, ly.wk_dt, D, range(k0, k1), 0, D, pk) ||
            !repack(ly.wv, ly.wv_dt, D, range(k0, k1), 0, D, pv)) {
            jdg_set_err(e->ctx, "layer %d q/k/v: dtype %d has no kernel for dim %d", l, ly.wq_dt, D);
            return JD_EUNSUPPORTED;
        }
        pqkv.dt = pq.dt;
        pqkv.rows = pq.rows + pk.rows + pv.rows;
        pqkv.cols = D;
        for (const Packed *x : {&pq, &pk, &pv}) {
            pqkv.q.insert(pqkv.q.end(), x->q.begin(), x->q.end());
            pqkv.s.insert(pqkv.s.end(), x->s.begin(), x->s.end());
        }
        // Wo: all rows, the contraction columns of this rank's heads
        if (!repack(ly.wo, ly.wo_dt, Hh * HD, range(0, D), q0, q1, po)) {
            jdg_set_err(e->ctx, "layer %d wo: dtype %d cannot be split at %d", l, ly.wo_dt, q0);
            return JD_EUNSUPPORTED;
        }
        // gate/up interleaved rows (g_i, u_i) of this rank's hidden slice
        const int h0 = sh.hidden0, h1 = h0 + sh.hidden;
        std::vector<int> gi = range(h0, h1);
        if (!repack(ly.gate, ly.gate_dt, D, gi, 0, D, pg) || !repack(ly.up, ly.up_dt, D, gi, 0, D, pu)) {
            jdg_set_err(e->ctx, "layer %d gate/up: dtype %d has no kernel", l, ly.gate_dt);
            return JD_EUNSUPPORTED;
        }
        {
            pgu.dt = pg.dt;
            pgu.rows = 2 * pg.rows;
            pgu.cols = D;
            const size_t qr = pg.q.size() / pg.rows, sr = pg.rows ? pg.s.size() / pg.rows : 0;
            pgu.q.resize(pg.q.size() * 2);
            pgu.s.resize(pg.s.size() * 2);
            for (int i = 0; i < pg.rows; i++) {
                memcpy(&pgu.q[(2 * i) * qr], &pg.q[i * qr], qr);
                memcpy(&pgu.q[(2 * i + 1) * qr], &pu.q[i * qr], qr);
                if (sr) {
                    memcpy(&pgu.s[(2 * i) * sr], &pg.s[i * sr], sr);
                    memcpy(&pgu.s[(2 * i + 1) * sr], &pu.s[i * sr], sr);
                }
            }
        }
        if (!repack(ly.down, ly.down_dt, HH, range(0, D), h0, h1, pd)) {
            jdg_set_err(e->ctx, "layer %d down: dtype %d cannot be split at %d", l, ly.down_dt, h0);
            return JD_EUNSUPPORTED;
        }
        int rc;
        if ((rc = upload_packed(e, pqkv, hp->wqkv[l])) || (rc = upload_packed(e, po, hp->wo[l])) ||
            (rc = upload_packed(e, pgu, hp->gu[l])) || (rc = upload_packed(e, pd, hp->dn[l])))
            return rc;
        HostLayerDev &hl = e->hl[l];
        if (ly.attn_norm) { if ((rc = upload_f32(e, ly.attn_norm, D, &hl.attn_norm))) return rc; }
        if (ly.ffn_norm) { if ((rc = upload_f32(e, ly.ffn_norm, D, &hl.ffn_norm))) return rc; }
        // LoRA parliament: vote rows, alive mask, A [16][D][R], B [16][R][D]
        if (!h->w_vote[l]) {
            jdg_set_err(e->ctx, "layer %d has no LoRA vote rows", l);
            return JD_EINVAL;
        }
        if ((rc = upload_f32(e, h->w_vote[l], (size_t)JD_MAX_EXPERTS * D, &hl.w_vote))) return rc;
        std::vector<float> A((size_t)JD_MAX_EXPERTS * D * R, 0.f), Bm((size_t)JD_MAX_EXPERTS * R * D, 0.f);
        std::vector<int> alive(JD_MAX_EXPERTS, 0);
        int na = 0;
        for (int x = 0; x < JD_MAX_EXPERTS; x++) {
            // an elected expert without factors is skipped by the reference (janusdoe.c:3289);
            // its slot is kept alive for the election with zero factors
            alive[x] = h->alive[l][x] ? 1 : 0;
            na += alive[x];
            if (alive[x] && h->A[l][x] && h->B[l][x]) {
                memcpy(&A[(size_t)x * D * R], h->A[l][x], (size_t)D * R * 4);
                memcpy(&Bm[(size_t)x * R * D], h->B[l][x], (size_t)R * D * 4);
            }
        }
        e->n_alive[l] = na;
        if ((rc = upload_f32(e, A.data(), A.size(), &hp->lora_A[l]))) return rc;
        if ((rc = upload_f32(e, Bm.data(), Bm.size(), &hp->lora_B[l]))) return rc;
        DALLOC(hl.alive, JD_MAX_EXPERTS * 4);
        CK(cudaMemcpy(hl.alive, alive.data(), JD_MAX_EXPERTS * 4, cudaMemcpyHostToDevice));
        hl.focus = h->layer_focus[l];
        hl.attn_bias = h->attention_bias[l];
        e->layer_consensus[l] = h->consensus0[l];
    }
    {
        int rc;
        std::vector<float> ones(D, 1.0f);
        if ((rc = upload_f32(e, ones.data(), D, &hp->ones))) return rc;
        if ((rc = upload_f32(e, h->tok_emb, (size_t)h->vocab * D, &e->tok_emb))) return rc;
        if (h->output_norm) { if ((rc = upload_f32(e, h->output_norm, D, &e->output_norm))) return rc; }
        else e->output_norm = hp->ones;
        Packed po;
        const void *outw = h->output;
        int odt = h->output_dt;
        if (!repack(outw, odt, D, range(hp->V_off, hp->V_off + hp->V_loc), 0, D, po)) {
            jdg_set_err(e->ctx, "output: dtype %d has no kernel", odt);
            return JD_EUNSUPPORTED;
        }
        if ((rc = upload_packed(e, po, hp->out))) return rc;
    }
    // RoPE table: ang = pos / powf(theta, 2i/HD) (janusdoe.c:3203)
    {
        const int half = HD / 2;
        std::vector<float> cs((size_t)max_seq * half), sn((size_t)max_seq * half);
        for (int p = 0; p < max_seq; p++)
            for (int i = 0; i < half; i++) {
                float ang = (float)p / powf(h->rope_theta, 2.0f * i / (float)HD);
                cs[(size_t)p * half + i] = cosf(ang);
                sn[(size_t)p * half + i] = sinf(ang);
            }
        int rc;
        if ((rc = upload_f32(e, cs.data(), cs.size(), &e->rope_cos))) return rc;
        if ((rc = upload_f32(e, sn.data(), sn.size(), &e->rope_sin))) return rc;
    }
    // activations and state
    const int B = max_batch;
    DALLOC(e->x, (size_t)B * D * 4);
    DALLOC(e->xn, (size_t)B * D * 4);
    DALLOC(e->xb, (size_t)B * D * 4);
    DALLOC(e->qkv, (size_t)B * e->qkvd * 4);
    DALLOC(e->att, (size_t)B * e->qd * 4);
    DALLOC(e->part, (size_t)B * e->Hh * e->nchunk * (HD + 2) * 4);
    DALLOC(e->hbuf, (size_t)B * e->hidden * 4);
    DALLOC(e->logits, (size_t)B * std::max(1, hp->V_loc) * 4);
    DALLOC(e->lora_t, (size_t)B * kMaxE * R * 4);
    DALLOC(hp->partial, (size_t)B * D * 4);
    DALLOC(hp->amx_v, (size_t)world * B * 4);
    DALLOC(hp->amx_i, (size_t)world * B * 4);
    DALLOC(hp->amx_v_loc, (size_t)B * 4);
    DALLOC(hp->amx_i_loc, (size_t)B * 4);
    e->kv_bstride = (long)L * max_seq * e->kd;
    DALLOC(e->kc, (size_t)B * e->kv_bstride * 4);
    DALLOC(e->vc, (size_t)B * e->kv_bstride * 4);
    {
        int dev = 0;
        CK(cudaGetDevice(&dev));
        CK(cudaDeviceGetAttribute(&hp->n_sm, cudaDevAttrMultiProcessorCount, dev));
    }
    if (max_batch > 1) {
        const int kmax = std::max(D, std::max(e->qd, e->hidden));
        if (kmax % 256 == 0) {
            DALLOC(hp->xprep, (size_t)(kmax / 256) * kQmBBytes);
            // split K only for matrices with fewer row tiles than SMs: rows < 148 * 128
            DALLOC(hp->qm_part, (size_t)kQmMaxSplit * kQmTok * 160 * kQmRows * 4);
            DALLOC(hp->qm_tickets, 1024 * 4);
            CK(cudaMemset(hp->qm_tickets, 0, 1024 * 4));
            // tensor maps of every Q4_K matrix the batched GEMM reads
            std::vector<const QW *> mats;
            for (int l = 0; l < L; l++) {
                mats.push_back(&hp->wqkv[l]);
                mats.push_back(&hp->wo[l]);
                mats.push_back(&hp->gu[l]);
                mats.push_back(&hp->dn[l]);
            }
            mats.push_back(&hp->out);
            for (const QW *w : mats)
                if (w->dt == JD_Q4_K && w->cols % 256 == 0 && w->rows > 0) {
                    const int rc = qm_add_maps(e, *w);
                    if (rc != JD_OK) return rc;
                }
        }
    }
    DALLOC(hp->votes, kMaxE * 4);
    DALLOC(hp->tall, (size_t)kMaxE * R * 4);
    if (max_batch > 1 && D % 256 == 0 && R % 4 == 0 && R <= 20) {
        DALLOC(hp->hpar_part, (size_t)(D / 256) * kMaxE * (R + 1) * kHparTok * 4);
        DALLOC(hp->hpar_tickets, (kMaxE + 1) * 4);
        CK(cudaMemset(hp->hpar_tickets, 0, (kMaxE + 1) * 4));
        DALLOC(hp->hpar_votes, (size_t)max_batch * kMaxE * 4);
        DALLOC(hp->hpar_tall, (size_t)max_batch * kMaxE * R * 4);
        CK(cudaStreamCreateWithFlags(&hp->st2, cudaStreamNonBlocking));
        hp->ev_fork.assign(L, nullptr);
        hp->ev_join.assign(L, nullptr);
        for (int l = 0; l < L; l++) {
            CK(cudaEventCreateWithFlags(&hp->ev_fork[l], cudaEventDisableTiming));
            CK(cudaEventCreateWithFlags(&hp->ev_join[l], cudaEventDisableTiming));
        }
    }
    DALLOC(e->amax_v, 1024 * 4);
    DALLOC(e->amax_i, 1024 * 4);
    for (int l = 0; l < L; l++) {
        std::vector<int> al;
        for (int x = 0; x < kMaxE; x++)
            if (h->alive[l][x]) al.push_back(x);
        al.resize(kMaxE, 0);
        DALLOC(hp->alive_list[l], kMaxE * 4);
        CK(cudaMemcpy(hp->alive_list[l], al.data(), kMaxE * 4, cudaMemcpyHostToDevice));
    }
    {
        // batch-1 chain: one GPU, packed Q8_0/Q4_K matrices with at most 16 code chunks per
        // row held in registers, head sizes the attention CTA handles, float4 vector loads
        bool ok = world == 1 && HD % 64 == 0 && HD <= 128 && hp->H_loc <= 64 && max_seq <= 1024 && D % 128 == 0 &&
                  e->qd % 128 == 0 && e->hidden % 64 == 0 && hb1_maxc(hp->out) > 0;
        for (int l = 0; l < L && ok; l++)
            ok = hb1_maxc(hp->wqkv[l]) > 0 && hb1_maxc(hp->wo[l]) > 0 && hb1_maxc(hp->gu[l]) > 0 &&
                 hb1_maxc(hp->dn[l]) > 0;
        hp->hb1 = ok;
        const char *g = getenv("JDG_GENERIC");
        e->force_generic = g && g[0] == '1';
        if (ok) {
            // persistent GU and LM grids: as many CTAs as stay resident on every SM
            int rc2 = jdg_host_set_attrs(e);
            if (rc2 != JD_OK) return rc2;
            int dev = 0, n_sm = 148;
            CK(cudaGetDevice(&dev));
            CK(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
            const size_t vec_sm = ((size_t)D + D / 16) * 4;
            hp->gu_ctas = hb1_resident(hp->gu[0], vec_sm, 0) * n_sm;
            hp->lm_ctas = hb1_resident(hp->out, vec_sm, 1) * n_sm;
            if (hp->gu_ctas < 1 || hp->lm_ctas < 1) {
                jdg_set_err(e->ctx, "batch-1 chain: occupancy query failed");
                return JD_ECUDA;
            }
            hp->lm_ctas = std::min(hp->lm_ctas, 1024);  // argmax partials
        }
    }
    int rc = jdg_alloc_state(e);
    if (rc != JD_OK) return rc;
    rc = jdg_reset(e, -1);
    if (rc != JD_OK) return rc;
    CK(cudaStreamSynchronize(e->st));
    return JD_OK;
}

// ------------------------------------------------------------------------------------
// C (epi)= W . X for M tokens.  do_norm: X is first RMS-normed with norm_w (null = ones,
// janusdoe.c:504), the normed rows also going to xn_out when given.
template <int EPI>
static void launch_q(jdg_engine *e, const QW &w, const float *X, int ldx, int M, float *C, int ldc, float alpha,
                     int do_norm = 0, const float *norm_w = nullptr, float *xn_out = nullptr) {
    const bool tc = M > 1 && w.dt == JD_Q4_K && w.cols % 256 == 0 && priv(e) && priv(e)->xprep;
    if (do_norm && !tc) {
        // the other paths read a normed copy
        float *dst = xn_out ? xn_out : e->xb;
        k_rmsnorm<<<M, 256, 0, e->st>>>(X, norm_w, dst, w.cols, e->eps);
        e->launches++;
        X = dst;
        ldx = w.cols;
    }
    if (M == 1) {
        QGemvArgs a{w, X, C, alpha};
        const int units = EPI == EPI_SWIGLU ? w.rows / 2 : w.rows;  // one unit per warp, 8 warps
        const int grid = (units + 7) / 8;
        const size_t sm = ((size_t)w.cols + w.cols / 16) * 4;
        switch (w.dt) {
        case JD_Q8_0: k_qgemv<8, EPI><<<grid, 256, sm, e->st>>>(a); break;
        case JD_Q4_K: k_qgemv<12, EPI><<<grid, 256, sm, e->st>>>(a); break;
        case JD_Q6_K: k_qgemv<14, EPI><<<grid, 256, sm, e->st>>>(a); break;
        default: k_qgemv<0, EPI><<<grid, 256, sm, e->st>>>(a); break;
        }
    } else if (tc) {
        // tensor cores (tcgen05): 32 tokens per launch
        const QmMaps *maps = qm_find_maps(e, w);
        if (!maps) {
            // the maps are made at upload for every matrix that can come here
            jdg_set_err(e->ctx, "tensor-core GEMM: no tensor maps for a %d x %d matrix", w.rows, w.cols);
            cudaMemsetAsync(e->err, 0xFF, sizeof(int), e->st);
            return;
        }
        for (int t0 = 0; t0 < M; t0 += kQmTok) {
            const int mt = std::min(kQmTok, M - t0);
            {
                // programmatic dependent launch: queued behind the previous kernel, it waits
                // for that grid before reading X
                cudaLaunchConfig_t pc = {};
                pc.gridDim = dim3(kQmTok);
                pc.blockDim = dim3(256);
                pc.stream = e->st;
                cudaLaunchAttribute pa[1];
                pa[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
                pa[0].val.programmaticStreamSerializationAllowed = 1;
                pc.attrs = pa;
                pc.numAttrs = 1;
                cudaLaunchKernelEx(&pc, k_qm_prep_tok, X + (size_t)t0 * ldx, ldx, mt, w.cols, do_norm, norm_w, e->eps,
                                   xn_out ? xn_out + (size_t)t0 * ldx : (float *)nullptr, priv(e)->xprep);
            }
            QmArgs q = {};
            q.w = w;
            q.xprep = priv(e)->xprep;
            q.M = mt;
            q.C = C + (size_t)t0 * ldc;
            q.ldc = ldc;
            q.epi = EPI;
            q.alpha = alpha;
            q.err = e->err;
            // split K across CTAs of a row tile until the tiles fill the SMs once (each split
            // keeps at least two superblocks)
            const int tiles = (w.rows + kQmRows - 1) / kQmRows, nsb = w.cols / 256;
            int ks = 1;
            if (tiles < priv(e)->n_sm) ks = std::max(1, std::min(std::min(priv(e)->n_sm / tiles, nsb / 2), kQmMaxSplit));
            q.ksplit = ks;
            q.part = priv(e)->qm_part;
            q.tickets = priv(e)->qm_tickets;
            // programmatic dependent launch: the GEMM's CTAs start while the prep kernel runs
            // (it triggers at once) and stream their first weight stages; they wait for it
            // before reading the prepared activations or C
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(tiles, ks);
            cfg.blockDim = dim3(kQmThreads);
            cfg.dynamicSmemBytes = kQmSmem;
            cfg.stream = e->st;
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            at[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = at;
            cfg.numAttrs = 1;
            cudaLaunchKernelEx(&cfg, k_qm_q4k, q, maps->codes, maps->hdr);
            e->launches += 2;
        }
        return;
    } else {
        QGemmArgs a{w, X, ldx, M, C, ldc, alpha};
        dim3 grid((w.rows + 63) / 64, (M + 31) / 32);
        const size_t sm = (size_t)(64 + 32) * 257 * 4;
        switch (w.dt) {
        case JD_Q8_0: k_qgemm<8, EPI><<<grid, 256, sm, e->st>>>(a); break;
        case JD_Q4_K: k_qgemm<12, EPI><<<grid, 256, sm, e->st>>>(a); break;
        case JD_Q6_K: k_qgemm<14, EPI><<<grid, 256, sm, e->st>>>(a); break;
        default: k_qgemm<0, EPI><<<grid, 256, sm, e->st>>>(a); break;
        }
    }
    e->launches++;
}

int jdg_host_set_attrs(jdg_engine *e) {
    (void)e;
    const int big = 200 * 1024;
#define SETA(K) cudaFuncSetAttribute(K, cudaFuncAttributeMaxDynamicSharedMemorySize, big)
    SETA((k_qgemv<8, EPI_STORE>)); SETA((k_qgemv<8, EPI_ADD>)); SETA((k_qgemv<8, EPI_SWIGLU>));
    SETA((k_qgemv<12, EPI_STORE>)); SETA((k_qgemv<12, EPI_ADD>)); SETA((k_qgemv<12, EPI_SWIGLU>));
    SETA((k_qgemv<14, EPI_STORE>)); SETA((k_qgemv<14, EPI_ADD>)); SETA((k_qgemv<14, EPI_SWIGLU>));
    SETA((k_qgemv<0, EPI_STORE>)); SETA((k_qgemv<0, EPI_ADD>)); SETA((k_qgemv<0, EPI_SWIGLU>));
    SETA((k_qgemm<8, EPI_STORE>)); SETA((k_qgemm<8, EPI_ADD>)); SETA((k_qgemm<8, EPI_SWIGLU>));
    SETA((k_qgemm<12, EPI_STORE>)); SETA((k_qgemm<12, EPI_ADD>)); SETA((k_qgemm<12, EPI_SWIGLU>));
    SETA((k_qgemm<14, EPI_STORE>)); SETA((k_qgemm<14, EPI_ADD>)); SETA((k_qgemm<14, EPI_SWIGLU>));
    SETA((k_qgemm<0, EPI_STORE>)); SETA((k_qgemm<0, EPI_ADD>)); SETA((k_qgemm<0, EPI_SWIGLU>));
    SETA((k_hb1_attn<64>)); SETA((k_hb1_attn<128>));
#define SETA_Q(K)                                                                                             \
    SETA((K<8, 4>)); SETA((K<8, 8>)); SETA((K<8, 12>)); SETA((K<8, 16>));                                     \
    SETA((K<12, 4>)); SETA((K<12, 8>)); SETA((K<12, 12>)); SETA((K<12, 16>));
    SETA_Q(k_hb1_qkv) SETA_Q(k_hb1_gu) SETA_Q(k_hb1_dn) SETA_Q(k_hb1_lm)
    SETA((k_hb1_wo<8, 4, 64>)); SETA((k_hb1_wo<8, 8, 64>)); SETA((k_hb1_wo<8, 12, 64>)); SETA((k_hb1_wo<8, 16, 64>));
    SETA((k_hb1_wo<12, 4, 64>)); SETA((k_hb1_wo<12, 8, 64>)); SETA((k_hb1_wo<12, 12, 64>));
    SETA((k_hb1_wo<12, 16, 64>));
    SETA((k_hb1_wo<8, 4, 128>)); SETA((k_hb1_wo<8, 8, 128>)); SETA((k_hb1_wo<8, 12, 128>));
    SETA((k_hb1_wo<8, 16, 128>));
    SETA((k_hb1_wo<12, 4, 128>)); SETA((k_hb1_wo<12, 8, 128>)); SETA((k_hb1_wo<12, 12, 128>));
    SETA((k_hb1_wo<12, 16, 128>));
#undef SETA_Q
#undef SETA
    if (cudaFuncSetAttribute(k_qm_q4k, cudaFuncAttributeMaxDynamicSharedMemorySize, kQmSmem) != cudaSuccess) {
        jdg_set_err(e->ctx, "cannot reserve %d bytes of shared memory for the tensor-core GEMM", kQmSmem);
        return JD_ECUDA;
    }
    if (cudaFuncSetAttribute(k_hpar_dots, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)hpar_dots_smem(20)) !=
            cudaSuccess ||
        cudaFuncSetAttribute(k_hpar_apply, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)hpar_apply_smem(kMaxE, 20)) !=
            cudaSuccess) {
        jdg_set_err(e->ctx, "cannot reserve shared memory for the parliament kernel");
        return JD_ECUDA;
    }
    return JD_OK;
}

// ------------------------------------------------------------------------------------
// Batch-1 chain launches (Programmatic Dependent Launch, jdg_hb1.cuh)
template <typename... KArgs, typename... Args>
static void hb1_launch(jdg_engine *e, void (*kern)(KArgs...), unsigned grid, size_t smem, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(128);
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
#define HB1_Q(KERN, QWV, GRID, SMEM, ARG)                                                          \
    switch ((QWV).dt * 100 + hb1_maxc(QWV)) {                                                      \
    case 804: hb1_launch(e, KERN<8, 4>, GRID, SMEM, ARG); break;                                  \
    case 808: hb1_launch(e, KERN<8, 8>, GRID, SMEM, ARG); break;                                  \
    case 812: hb1_launch(e, KERN<8, 12>, GRID, SMEM, ARG); break;                                 \
    case 816: hb1_launch(e, KERN<8, 16>, GRID, SMEM, ARG); break;                                 \
    case 1204: hb1_launch(e, KERN<12, 4>, GRID, SMEM, ARG); break;                                \
    case 1208: hb1_launch(e, KERN<12, 8>, GRID, SMEM, ARG); break;                                \
    case 1212: hb1_launch(e, KERN<12, 12>, GRID, SMEM, ARG); break;                               \
    default: hb1_launch(e, KERN<12, 16>, GRID, SMEM, ARG); break;                                 \
    }
#define HB1_WO(HDV, QWV, GRID, SMEM, ARG)                                                          \
    switch ((QWV).dt * 100 + hb1_maxc(QWV)) {                                                      \
    case 804: hb1_launch(e, k_hb1_wo<8, 4, HDV>, GRID, SMEM, ARG); break;                         \
    case 808: hb1_launch(e, k_hb1_wo<8, 8, HDV>, GRID, SMEM, ARG); break;                         \
    case 812: hb1_launch(e, k_hb1_wo<8, 12, HDV>, GRID, SMEM, ARG); break;                        \
    case 816: hb1_launch(e, k_hb1_wo<8, 16, HDV>, GRID, SMEM, ARG); break;                        \
    case 1204: hb1_launch(e, k_hb1_wo<12, 4, HDV>, GRID, SMEM, ARG); break;                       \
    case 1208: hb1_launch(e, k_hb1_wo<12, 8, HDV>, GRID, SMEM, ARG); break;                       \
    case 1212: hb1_launch(e, k_hb1_wo<12, 12, HDV>, GRID, SMEM, ARG); break;                      \
    default: hb1_launch(e, k_hb1_wo<12, 16, HDV>, GRID, SMEM, ARG); break;                        \
    }

static void enqueue_host_step_hb1(jdg_engine *e) {
    HostPriv *hp = priv(e);
    const int D = e->D, L = e->L, HD = e->HD, R = e->lora_rank;
    int n_sm = 148, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    HB1Args a = {};
    a.D = D; a.H = e->Hh; a.KVH = e->KVH; a.HD = HD; a.qd = e->qd; a.kd = e->kd; a.qkvd = e->qkvd;
    a.hidden = e->hidden; a.V = e->V; a.max_seq = e->max_seq; a.L = L; a.R = R;
    a.eps = e->eps; a.lora_alpha = e->lora_alpha;
    a.tok_emb = e->tok_emb; a.tok = e->tok; a.pos = e->pos;
    a.x = e->x; a.xn = e->xn;
    a.votes = hp->votes; a.tall = hp->tall;
    a.kcnt = e->kcnt; a.sel = e->sel; a.selw = e->selw; a.consensus = e->consensus;
    a.tr_k = e->tr_k; a.tr_sel = e->tr_sel; a.tr_w = e->tr_w; a.tr_ema = e->tr_ema;
    a.part = e->part;
    a.tickets = e->tickets; a.amax_v = e->amax_v; a.amax_i = e->amax_i;
    a.tok_out = e->tok; a.plen = e->plen; a.prompt = e->prompt; a.hist = e->hist; a.hist_n = e->hist_n;
    a.next_out = e->next_out; a.Hmax = e->Hmax; a.greedy_pick = e->temp <= 0.f;
    a.stats = e->stats; a.err = e->err; a.tl = e->timeline;
    // the attention CTAs take the own-model chain's arguments
    B1Args ab = {};
    ab.H = e->Hh; ab.KVH = e->KVH; ab.HD = HD; ab.qd = e->qd; ab.kd = e->kd; ab.max_seq = e->max_seq;
    ab.rope_norm = e->rope_norm; ab.rope_cos = e->rope_cos; ab.rope_sin = e->rope_sin;
    ab.clamp = 0.f; ab.inv_clamp = 0.f;
    ab.pos = e->pos; ab.qkv = e->qkv; ab.part = e->part; ab.err = e->err;
    const int nch = (e->max_seq + kB1Chunk - 1) / kB1Chunk;
    const size_t vec_sm = ((size_t)D + D / 16) * 4;
    const size_t attn_sm = (size_t)2 * kB1Chunk * (HD + 4) * 4;
    for (int l = 0; l < L; l++) {
        HostLayerDev &hl = e->hl[l];
        a.l = l;
        a.embed = l == 0;
        a.focus = hl.focus;
        a.w_vote = hl.w_vote; a.lora_A = hp->lora_A[l]; a.lora_B = hp->lora_B[l];
        a.alive = hl.alive; a.alive_list = hp->alive_list[l]; a.n_alive = e->n_alive[l];
        // QKV
        a.w = hp->wqkv[l];
        a.norm = hl.attn_norm ? hl.attn_norm : hp->ones;
        a.y = e->qkv;
        HB1_Q(k_hb1_qkv, a.w, (unsigned)((e->qkvd + 3) / 4), vec_sm, a);
        // ATTN (+ votes and LoRA projections)
        ab.l = l;
        ab.kc = e->kc + (size_t)l * e->max_seq * e->kd;
        ab.vc = e->vc + (size_t)l * e->max_seq * e->kd;
        ab.scale = (1.0f / sqrtf((float)HD)) * (1.0f + hl.attn_bias);
        a.natt = nch * e->KVH;
        const unsigned naux = (unsigned)((kMaxE + e->n_alive[l] * R + 3) / 4);
        if (HD == 64) hb1_launch(e, k_hb1_attn<64>, (unsigned)a.natt + naux, attn_sm, ab, a);
        else hb1_launch(e, k_hb1_attn<128>, (unsigned)a.natt + naux, attn_sm, ab, a);
        // WO (+ election CTA)
        a.w = hp->wo[l];
        const size_t wo_sm = ((size_t)e->qd + e->qd / 16) * 4;
        if (HD == 64) { HB1_WO(64, a.w, (unsigned)((D + 3) / 4), wo_sm, a); }
        else { HB1_WO(128, a.w, (unsigned)((D + 3) / 4), wo_sm, a); }
        // GU
        a.w = hp->gu[l];
        a.norm = hl.ffn_norm ? hl.ffn_norm : hp->ones;
        a.y = e->hbuf;
        HB1_Q(k_hb1_gu, a.w, (unsigned)(1 + hp->gu_ctas), vec_sm, a);
        // DN (+ LoRA deltas)
        a.w = hp->dn[l];
        a.hin = e->hbuf;
        HB1_Q(k_hb1_dn, a.w, (unsigned)((D + 3) / 4), ((size_t)e->hidden + e->hidden / 16) * 4, a);
    }
    a.w = hp->out;
    a.norm = e->output_norm;
    a.y = e->logits;
    a.embed = 0;
    HB1_Q(k_hb1_lm, a.w, (unsigned)hp->lm_ctas, vec_sm, a);
    if (!a.greedy_pick) jdg_launch_pick(e, 1);
}

// One decode step of gguf_host_forward (janusdoe.c:3160-3322) for slots 0..B-1.
int jdg_enqueue_host_step(jdg_engine *e, int B) {
    HostPriv *hp = priv(e);
    if (B == 1 && hp->hb1 && !e->force_generic) {
        enqueue_host_step_hb1(e);
        return JD_OK;
    }
    const int D = e->D, L = e->L;
    const bool tp = hp->world > 1;
    const float scale = 1.0f / sqrtf((float)e->HD);
    k_embed<<<B, 256, 0, e->st>>>(e->tok_emb, e->V, D, e->tok, e->x, e->err);
    e->launches++;
    const bool hpar = hp->hpar_part && B <= kHparTok;
    for (int l = 0; l < L; l++) {
        HostLayerDev &hl = e->hl[l];
        const bool hpar_l = hpar && e->n_alive[l] > 0;
        HParArgs pa = {};
        if (hpar_l) {
            pa.D = D; pa.R = e->lora_rank; pa.B = B; pa.L = L; pa.l = l;
            pa.xn = e->xn; pa.w_vote = hl.w_vote; pa.lora_A = hp->lora_A[l]; pa.lora_B = hp->lora_B[l];
            pa.alive = hl.alive; pa.alive_list = hp->alive_list[l]; pa.n_alive = e->n_alive[l];
            pa.part = hp->hpar_part; pa.tickets = hp->hpar_tickets;
            pa.votes = hp->hpar_votes; pa.tall = hp->hpar_tall;
            pa.kcnt = e->kcnt; pa.sel = e->sel; pa.selw = e->selw; pa.consensus = e->consensus;
            pa.tr_k = e->tr_k; pa.tr_sel = e->tr_sel; pa.tr_w = e->tr_w; pa.tr_ema = e->tr_ema;
            pa.lora_alpha = e->lora_alpha; pa.x = e->x;
        }
        launch_q<EPI_STORE>(e, hp->wqkv[l], e->x, D, B, e->qkv, e->qkvd, 1.f, 1, hl.attn_norm, e->xn);
        if (hpar_l) {
            // LoRA parliament, first half (janusdoe.c:3281-3293): votes, projections and
            // elections from xn, beside the rest of the layer
            CK(cudaEventRecord(hp->ev_fork[l], e->st));
            CK(cudaStreamWaitEvent(hp->st2, hp->ev_fork[l], 0));
            k_hpar_dots<<<dim3(D / 256, e->n_alive[l]), 256, hpar_dots_smem(pa.R), hp->st2>>>(pa);
            CK(cudaEventRecord(hp->ev_join[l], hp->st2));
            e->launches++;
        }
        jdg_launch_rope(e, l, B);
        jdg_launch_attention(e, l, B, scale, 1.0f + hl.attn_bias);
        if (!tp) {
            launch_q<EPI_ADD>(e, hp->wo[l], e->att, e->qd, B, e->x, D, 1.f);
        } else {
            launch_q<EPI_STORE>(e, hp->wo[l], e->att, e->qd, B, hp->partial, D, 1.f);
            ncclAllReduce(hp->partial, hp->partial, (size_t)B * D, ncclFloat, ncclSum, hp->comm, e->st);
            k_add<<<(unsigned)(((size_t)B * D + 255) / 256), 256, 0, e->st>>>(e->x, hp->partial, (size_t)B * D);
            e->launches++;
        }
        launch_q<EPI_SWIGLU>(e, hp->gu[l], e->x, D, B, e->hbuf, e->hidden, 1.f, 1, hl.ffn_norm);
        if (!tp && hp->learn_on && l == L - 1) {
            // the learning target dy is the last layer's FFN output (janusdoe.c:3274): kept,
            // then added to the residual exactly as the fused epilogue would
            launch_q<EPI_STORE>(e, hp->dn[l], e->hbuf, e->hidden, B, hp->learn_dyraw, D, 1.f);
            k_add_scaled<<<(D + 255) / 256, 256, 0, e->st>>>(e->x, hp->learn_dyraw, hl.focus, D);
            e->launches++;
        } else if (!tp) {
            launch_q<EPI_ADD>(e, hp->dn[l], e->hbuf, e->hidden, B, e->x, D, hl.focus);
        } else {
            launch_q<EPI_STORE>(e, hp->dn[l], e->hbuf, e->hidden, B, hp->partial, D, 1.f);
            ncclAllReduce(hp->partial, hp->partial, (size_t)B * D, ncclFloat, ncclSum, hp->comm, e->st);
            k_add<<<(unsigned)(((size_t)B * D + 255) / 256), 256, 0, e->st>>>(e->x, hp->partial, (size_t)B * D);
            e->launches++;
        }
        // LoRA parliament on xn (janusdoe.c:3281-3303)
        if (hpar_l) {
            CK(cudaStreamWaitEvent(e->st, hp->ev_join[l], 0));
            k_hpar_apply<<<(D + 31) / 32, 256, hpar_apply_smem(e->n_alive[l], pa.R), e->st>>>(pa);
            e->launches++;
            continue;
        }
        jdg_launch_elect(e, l, B, e->xn, nullptr, hl.w_vote, hl.alive, 0.f, 1);
        if (e->n_alive[l] > 0) {
            k_lora_t<<<dim3(e->lora_rank, e->n_alive[l], B), 256, 0, e->st>>>(hp->lora_B[l], e->lora_rank, D, e->kcnt,
                                                                              e->sel, e->xn, e->lora_t);
            k_lora_apply<<<dim3((D + 255) / 256, B), 256, 0, e->st>>>(hp->lora_A[l], e->lora_rank, D, e->lora_alpha,
                                                                      e->kcnt, e->sel, e->selw, e->lora_t, e->x);
            e->launches += 2;
        }
    }
    if (!tp) {
        launch_q<EPI_STORE>(e, hp->out, e->x, D, B, e->logits, hp->V_loc, 1.f, 1, e->output_norm);
        if (hp->learn_on) {
            // the normed final hidden is in xb (janusdoe.c:3311): both targets RMS-normalised,
            // then the signal of the next token from the logits
            k_learn_capture<<<1, 1024, 0, e->st>>>(e->xb, hp->learn_dyraw, D, hp->learn_x, hp->learn_dy);
            k_learn_signal<<<1, 1024, 0, e->st>>>(e->logits, hp->V_loc, hp->learn_next, hp->learn_sig);
            e->launches += 2;
        }
        jdg_launch_pick(e, B);
    } else {
        launch_q<EPI_STORE>(e, hp->out, e->x, D, B, e->logits, hp->V_loc, 1.f, 1, e->output_norm);
        k_argmax_part<<<B, 1024, 0, e->st>>>(e->logits, hp->V_loc, hp->V_loc, hp->V_off, hp->amx_v_loc, hp->amx_i_loc);
        ncclAllGather(hp->amx_v_loc, hp->amx_v, B, ncclFloat, hp->comm, e->st);
        ncclAllGather(hp->amx_i_loc, hp->amx_i, B, ncclInt32, hp->comm, e->st);
        jdg_launch_pick_tp(e, B, hp->amx_v, hp->amx_i, hp->world);
        e->launches++;
    }
    return JD_OK;
}

void jdg_host_release(jdg_engine *e) {
    HostPriv *hp = priv(e);
    if (!hp) return;
    if (hp->comm) ncclCommDestroy(hp->comm);
    for (cudaEvent_t ev : hp->ev_fork)
        if (ev) cudaEventDestroy(ev);
    for (cudaEvent_t ev : hp->ev_join)
        if (ev) cudaEventDestroy(ev);
    if (hp->st2) cudaStreamDestroy(hp->st2);
    delete hp;
    e->host_priv = nullptr;
}

int jdg_engine_create(jdg_ctx *ctx, int kind, jdg_engine **out);

extern "C" int jdg_host_upload(jdg_ctx *ctx, const jd_host_model *h, int max_batch, int max_seq, jdg_engine **out) {
    return jdg_host_upload_tp(ctx, h, max_batch, max_seq, 0, 1, nullptr, out);
}

extern "C" int jdg_comm_unique_id(void *id) {
    if (!id) return JD_EINVAL;
    ncclUniqueId u;
    if (ncclGetUniqueId(&u) != ncclSuccess) return JD_ECOMM;
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
    memcpy(id, &u, 128);
    return JD_OK;
}

extern "C" int jdg_host_upload_tp(jdg_ctx *ctx, const jd_host_model *h, int max_batch, int max_seq, int rank, int world,
                                  const void *id, jdg_engine **out) {
    if (!ctx || !h || !out || max_batch < 1 || max_batch > 4096 || max_seq < 1 || world < 1 || rank < 0 ||
        rank >= world || (world > 1 && !id) || !h->tok_emb || h->n_layers < 1) {
        if (ctx) jdg_set_err(ctx, "jdg_host_upload: bad arguments");
        return JD_EINVAL;
    }
    if ((h->head_dim != 64 && h->head_dim != 128) || h->n_kv_heads < 1 || h->n_heads % h->n_kv_heads ||
        h->n_heads / h->n_kv_heads > kMaxHG || h->dim % 32 || h->lora_rank < 1 || h->lora_rank > 64) {
        jdg_set_err(ctx, "jdg_host_upload: unsupported shape (dim %d heads %d/%d hd %d rank %d)", h->dim, h->n_heads,
                    h->n_kv_heads, h->head_dim, h->lora_rank);
        return JD_EUNSUPPORTED;
    }
    jdg_engine *e = nullptr;
    int rc = jdg_engine_create(ctx, 1, &e);
    if (rc != JD_OK) return rc;
    e->host_priv = new (std::nothrow) HostPriv();
    if (!e->host_priv) {
        jdg_engine_free(e);
        return JD_ENOMEM;
    }
    if (world > 1) {
        ncclUniqueId u;
        memcpy(&u, id, 128);
        ncclResult_t r = ncclCommInitRank(&priv(e)->comm, world, u, rank);
        if (r != ncclSuccess) {
            jdg_set_err(ctx, "ncclCommInitRank(%d of %d): %s", rank, world, ncclGetErrorString(r));
            jdg_engine_free(e);
            return JD_ECOMM;
        }
    }
    rc = host_upload_impl(e, h, max_batch, max_seq, rank, world);
    if (rc != JD_OK) {
        jdg_engine_free(e);
        return rc;
    }
    *out = e;
    return JD_OK;
}

// ------------------------------------------------------------------------------------
// Hebbian --learn pass (janusdoe.c:3416-3447) on the engine's LoRA parliament.
static float learn_uniform(uint64_t *s) {  // janusdoe.c:191-192
    uint64_t x = *s;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    *s = x;
    return (float)(x & 0x7FFFFFFFull) / (float)0x7FFFFFFF;
}
static float learn_normal(uint64_t *s) {  // janusdoe.c:193 (host libm, as the reference)
    float u1 = learn_uniform(s), u2 = learn_uniform(s);
    if (u1 < 1e-10f) u1 = 1e-10f;
    return sqrtf(-2.0f * logf(u1)) * cosf(6.2831853f * u2);
}

static int learn_alloc(jdg_engine *e) {
    HostPriv *hp = priv(e);
    if (hp->learn_x) return JD_OK;
    const int D = e->D, L = e->L;
    DALLOC(hp->learn_dyraw, (size_t)D * 4);
    DALLOC(hp->learn_x, (size_t)D * 4);
    DALLOC(hp->learn_dy, (size_t)D * 4);
    DALLOC(hp->learn_sig, 4);
    DALLOC(hp->learn_next, 4);
    DALLOC(hp->learn_dead, (size_t)L * JD_MAX_EXPERTS * 4);
    DALLOC(hp->learn_upd, (size_t)L * JD_MAX_EXPERTS * sizeof(LearnUpd));
    DALLOC(hp->learn_A, (size_t)L * sizeof(float *));
    DALLOC(hp->learn_B, (size_t)L * sizeof(float *));
    DALLOC(hp->learn_alive, (size_t)L * sizeof(int *));
    std::vector<float *> pa(L), pb(L);
    std::vector<int *> pl(L);
    for (int l = 0; l < L; l++) {
        pa[l] = hp->lora_A[l];
        pb[l] = hp->lora_B[l];
        pl[l] = e->hl[l].alive;
    }
    CK(cudaMemcpy(hp->learn_A, pa.data(), L * sizeof(float *), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(hp->learn_B, pb.data(), L * sizeof(float *), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(hp->learn_alive, pl.data(), L * sizeof(int *), cudaMemcpyHostToDevice));
    return JD_OK;
}

int jdg_reset(jdg_engine *e, int slot);
int jdg_host_drop_graphs(jdg_engine *e);

extern "C" int jdg_host_learn(jdg_engine *e, const int *toks, int nt, float lr, uint64_t *rng, int *notorch_offset,
                              int *deaths) {
    if (!e || !toks || nt < 1 || !rng || !notorch_offset || e->kind != 1 || !priv(e)) return JD_EINVAL;
    HostPriv *hp = priv(e);
    if (hp->world != 1 || e->lora_rank < 1) {
        jdg_set_err(e->ctx, "jdg_host_learn: one GPU and a LoRA parliament are needed");
        return JD_EUNSUPPORTED;
    }
    cudaSetDevice(jdg_ctx_device(e->ctx));
    int rc = learn_alloc(e);
    if (rc != JD_OK) return rc;
    const int L = e->L, D = e->D, R = e->lora_rank, nr = R < kLearnLanes ? R : kLearnLanes;
    // fresh caches for slot 0 (the reference allocates them per pass); the EMA carries on
    const size_t kv = (size_t)L * e->max_seq * e->kd * 4;
    CK(cudaMemsetAsync(e->kc, 0, kv, e->st));
    CK(cudaMemsetAsync(e->vc, 0, kv, e->st));
    std::vector<int> alive((size_t)L * JD_MAX_EXPERTS);
    for (int l = 0; l < L; l++)
        CK(cudaMemcpyAsync(&alive[(size_t)l * JD_MAX_EXPERTS], e->hl[l].alive, JD_MAX_EXPERTS * 4,
                           cudaMemcpyDeviceToHost, e->st));
    CK(cudaStreamSynchronize(e->st));
    const int saved_generic = e->force_generic;
    e->force_generic = 1;  // the generic step carries the learning captures
    hp->learn_on = true;
    int killed = 0, err_rc = JD_OK;
    std::vector<int> tr_k(L), tr_sel((size_t)L * kMaxE), dead;
    std::vector<LearnUpd> upd;
    for (int t = 0; t + 1 < nt && t < e->max_seq - 1; t++) {
        int io[3] = {toks[t], t, toks[t + 1]};
        CK(cudaMemcpyAsync(e->tok, &io[0], 4, cudaMemcpyHostToDevice, e->st));
        CK(cudaMemcpyAsync(e->pos, &io[1], 4, cudaMemcpyHostToDevice, e->st));
        CK(cudaMemcpyAsync(hp->learn_next, &io[2], 4, cudaMemcpyHostToDevice, e->st));
        err_rc = jdg_enqueue_host_step(e, 1);
        if (err_rc != JD_OK) break;
        float sig = 0.f;
        CK(cudaMemcpyAsync(&sig, hp->learn_sig, 4, cudaMemcpyDeviceToHost, e->st));
        CK(cudaMemcpyAsync(tr_k.data(), e->tr_k, (size_t)L * 4, cudaMemcpyDeviceToHost, e->st));
        CK(cudaMemcpyAsync(tr_sel.data(), e->tr_sel, (size_t)L * kMaxE * 4, cudaMemcpyDeviceToHost, e->st));
        CK(cudaStreamSynchronize(e->st));
        // the experts elected in this token, layer by layer, slot by slot (janusdoe.c:3437-3445)
        upd.clear();
        if (fabsf(sig) >= 1e-8f) {
            for (int l = 0; l < L; l++)
                for (int x = 0; x < JD_MAX_EXPERTS; x++) {
                    if (!alive[(size_t)l * JD_MAX_EXPERTS + x]) continue;
                    bool elected = false;
                    for (int q = 0; q < tr_k[l]; q++) elected |= tr_sel[(size_t)l * kMaxE + q] == x;
                    if (!elected) continue;
                    LearnUpd u;
                    u.l = l;
                    u.e = x;
                    u.base = *notorch_offset % R;
                    for (int j = 0; j < kLearnLanes; j++) u.noise[j] = j < nr ? learn_normal(rng) : 0.f;
                    *notorch_offset = (u.base + nr) % R;
                    upd.push_back(u);
                }
        }
        if (!upd.empty()) {
            float s = sig > 2.0f ? 2.0f : sig < -2.0f ? -2.0f : sig;
            LearnArgs a;
            a.upd = hp->learn_upd; a.A = hp->learn_A; a.B = hp->learn_B; a.alive = hp->learn_alive;
            a.x = hp->learn_x; a.dy = hp->learn_dy; a.D = D; a.R = R; a.nr = nr; a.lr = lr * s; a.dead = hp->learn_dead;
            CK(cudaMemcpyAsync(hp->learn_upd, upd.data(), upd.size() * sizeof(LearnUpd), cudaMemcpyHostToDevice, e->st));
            k_learn_update<<<(unsigned)upd.size(), 256, 0, e->st>>>(a);
            e->launches++;
            dead.assign(upd.size(), 0);
            CK(cudaMemcpyAsync(dead.data(), hp->learn_dead, dead.size() * 4, cudaMemcpyDeviceToHost, e->st));
            CK(cudaStreamSynchronize(e->st));
            for (size_t m = 0; m < upd.size(); m++)
                if (dead[m]) {  // quarantined: the kernel cleared its alive flag on the device
                    alive[(size_t)upd[m].l * JD_MAX_EXPERTS + upd[m].e] = 0;
                    killed++;
                }
        }
    }
    hp->learn_on = false;
    e->force_generic = saved_generic;
    if (killed) {
        // elections, the chain and the batched parliament read the alive lists
        for (int l = 0; l < L; l++) {
            std::vector<int> al;
            for (int x = 0; x < JD_MAX_EXPERTS; x++)
                if (alive[(size_t)l * JD_MAX_EXPERTS + x]) al.push_back(x);
            e->n_alive[l] = (int)al.size();
            al.resize(kMaxE, 0);
            if (hp->alive_list[l]) CK(cudaMemcpy(hp->alive_list[l], al.data(), kMaxE * 4, cudaMemcpyHostToDevice));
        }
        jdg_host_drop_graphs(e);
    }
    if (deaths) *deaths = killed;
    if (err_rc != JD_OK) return err_rc;
    CK(cudaStreamSynchronize(e->st));
    return JD_OK;
}

// A [D][R], B [R][D] and the alive flag of LoRA expert slot x of layer l
extern "C" int jdg_host_get_expert(jdg_engine *e, int l, int x, float *A, float *B, int *alive) {
    if (!e || e->kind != 1 || !priv(e) || l < 0 || l >= e->L || x < 0 || x >= JD_MAX_EXPERTS) return JD_EINVAL;
    HostPriv *hp = priv(e);
    cudaSetDevice(jdg_ctx_device(e->ctx));
    const size_t n = (size_t)e->D * e->lora_rank;
    if (A) CK(cudaMemcpy(A, hp->lora_A[l] + (size_t)x * n, n * 4, cudaMemcpyDeviceToHost));
    if (B) CK(cudaMemcpy(B, hp->lora_B[l] + (size_t)x * n, n * 4, cudaMemcpyDeviceToHost));
    if (alive) CK(cudaMemcpy(alive, e->hl[l].alive + x, 4, cudaMemcpyDeviceToHost));
    return JD_OK;
}

// ------------------------------------------------------------------------------------
// Standalone packed GEMV/GEMM through host buffers (jd_qmatvec, janusdoe.c:2685).
extern "C" int jdg_qmatvec(jdg_ctx *ctx, float *out, const void *W, int dt, const float *x, int r, int c, int B) {
    if (!ctx || !out || !W || !x || r < 1 || c < 1 || B < 1) return JD_EINVAL;
    const int be = block_elems(dt);
    if (!be || c % be) {
        jdg_set_err(ctx, "jdg_qmatvec: dtype %d with %d columns has no kernel", dt, c);
        return JD_EUNSUPPORTED;
    }
    if (dt == JD_Q4_K && c % 256) return JD_EUNSUPPORTED;
    if (dt == JD_F32 && c % 4) return JD_EUNSUPPORTED;
    if (B > 1 && c % 256) {
        jdg_set_err(ctx, "jdg_qmatvec: batched product needs columns in multiples of 256");
        return JD_EUNSUPPORTED;
    }
    jdg_engine *e = nullptr;
    int rc = jdg_engine_create(ctx, 1, &e);
    if (rc != JD_OK) return rc;
    Packed p;
    if (!repack(W, dt, c, range(0, r), 0, c, p)) {
        jdg_engine_free(e);
        return JD_EUNSUPPORTED;
    }
    QW w;
    float *dx = nullptr, *dy = nullptr;
    rc = upload_packed(e, p, w);
    if (rc == JD_OK && dt == JD_Q4_K && B > 1) {
        // batched Q4_K products run on the tensor cores, as in the engine
        e->host_priv = new (std::nothrow) HostPriv();
        HostPriv *hp = priv(e);
        if (!hp) rc = JD_ENOMEM;
        if (rc == JD_OK) {
            int dev = 0;
            cudaGetDevice(&dev);
            cudaDeviceGetAttribute(&hp->n_sm, cudaDevAttrMultiProcessorCount, dev);
            rc = dalloc(e, (void **)&hp->xprep, (size_t)(c / 256) * kQmBBytes);
        }
        if (rc == JD_OK) rc = dalloc(e, (void **)&hp->qm_part, (size_t)kQmMaxSplit * kQmTok * 160 * kQmRows * 4);
        if (rc == JD_OK) rc = dalloc(e, (void **)&hp->qm_tickets, 1024 * 4);
        if (rc == JD_OK && cudaMemset(hp->qm_tickets, 0, 1024 * 4) != cudaSuccess) rc = JD_ECUDA;
        if (rc == JD_OK) rc = qm_add_maps(e, w);
    }
    if (rc == JD_OK) rc = dalloc(e, (void **)&dx, (size_t)B * c * 4);
    if (rc == JD_OK) rc = dalloc(e, (void **)&dy, (size_t)B * r * 4);
    if (rc == JD_OK) rc = jdg_host_set_attrs(e);
    if (rc == JD_OK) {
        cudaError_t ce = cudaMemcpy(dx, x, (size_t)B * c * 4, cudaMemcpyHostToDevice);
        if (ce == cudaSuccess) {
            launch_q<EPI_STORE>(e, w, dx, c, B, dy, r, 1.f);
            ce = cudaStreamSynchronize(e->st);
        }
        if (ce == cudaSuccess) ce = cudaMemcpy(out, dy, (size_t)B * r * 4, cudaMemcpyDeviceToHost);
        if (ce != cudaSuccess) {
            jdg_set_err(ctx, "jdg_qmatvec: %s", cudaGetErrorString(ce));
            rc = JD_ECUDA;
        }
    }
    jdg_engine_free(e);
    return rc;
}

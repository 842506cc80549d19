// qw_model.cu -- the C ABI of libqwen3_b200.so: model object, weight placement and sharding,
// paged KV cache, and the decode / prefill / generate schedules.
//
// Stands in for the reference's compiled Qwen3 graph (engine/ml/src/main/java/org/almostrealism/ml/
// qwen3/Qwen3.java:334-415 built into CompiledModel, CompiledModel.java:271-341) and the
// AutoregressiveModel loop around it (AutoregressiveModel.java:295-308, 405-434).
#include <cuda_runtime.h>
#include <nccl.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <algorithm>
#include <string>
#include <vector>

#include "../../include/qwen3_b200.h"
#include "qw_kernels.h"
#include "qw_prefill.h"
#include "qw_ops.h"
#include "qw_tc.h"
#include "qw_ar.h"

using namespace qw;

namespace {

enum Kind {
    K_EMBED = 0, K_LMHEAD = 1, K_NORM = 2, K_FREQ = 3,
    K_RMS_ATT = 0, K_RMS_FFN, K_WQ, K_WK, K_WV, K_WO, K_BQ, K_BK, K_BV, K_QN, K_KN, K_W1, K_W3, K_W2, K_NUM_LAYER_KINDS
};
const char *kLayerNames[K_NUM_LAYER_KINDS] = {
    "input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_proj.weight", "self_attn.k_proj.weight",
    "self_attn.v_proj.weight", "self_attn.o_proj.weight", "self_attn.q_proj.bias", "self_attn.k_proj.bias",
    "self_attn.v_proj.bias", "self_attn.q_norm.weight", "self_attn.k_norm.weight", "mlp.gate_proj.weight",
    "mlp.up_proj.weight", "mlp.down_proj.weight"};

struct Layer {
    void *w_qkv = nullptr;   // (Ql + 2 KVl, D)
    float *b_qkv = nullptr;  // (Ql + 2 KVl)
    float *qn = nullptr, *kn = nullptr;  // (Ql), (KVl)
    void *w_o = nullptr;     // (D, Ql)
    void *w_gu = nullptr;    // (2 Fl, D) gate/up interleaved in blocks of 16 rows
    void *w_down = nullptr;  // (D, Fl)
    float *rms_att = nullptr, *rms_ffn = nullptr;
    uint32_t loaded = 0;
};

}  // namespace

struct qw_model {
    qw_config c{};
    int dev = 0, rank = 0, tp = 1, num_sms = 148;
    cudaStream_t st = nullptr;
    ncclComm_t comm = nullptr;
    bool bf16w = false, bf16kv = false;
    size_t wsz = 4, kvsz = 4;
    int D = 0, Hl = 0, Hkvl = 0, Ql = 0, KVl = 0, Fl = 0, Vl = 0, v0 = 0, QKVl = 0;
    std::vector<Layer> L;
    void *embed = nullptr, *lm = nullptr;
    bool lm_alias = false;
    float *norm_final = nullptr;
    uint32_t top_loaded = 0;
    bool finalized = false;
    float2 *freq = nullptr;
    // paged KV
    int page_size = 64, log2_page = 6, num_pages = 0, max_pages = 0;
    void *kpool = nullptr, *vpool = nullptr;
    size_t layer_kv_elems = 0;
    int *d_page_table = nullptr;
    std::vector<int> h_page_table, free_pages;
    std::vector<std::vector<int>> slot_pages;
    // activations
    int T = 0, B = 0, maxsplit = 64;
    float *xa = nullptr, *xb = nullptr, *part = nullptr, *qkv = nullptr, *attn = nullptr, *hbuf = nullptr;
    float *part_o = nullptr, *part_ml = nullptr, *qk_ss = nullptr;
    unsigned *counters = nullptr, *am_counter = nullptr;
    float *logits = nullptr, *logits_all = nullptr, *am_pval = nullptr, *am_val = nullptr, *am_val_all = nullptr;
    int *am_pidx = nullptr, *am_idx = nullptr, *am_idx_all = nullptr;
    int *d_tokens = nullptr, *d_pos = nullptr, *d_slots = nullptr, *d_argmax = nullptr, *d_hist = nullptr;
    int hist_ld = 0;
    int *h_pin_i = nullptr;  // pinned staging: tokens | positions | slots | argmax
    PrefillBuffers pf{};
    bool tc_attn = false;  // prefill attention on tcgen05 (head_dim 128)
    // persistent batch-1 step kernel
    bool use_step = false;
    StepArgs step{};
    StepLayer *d_step_layers = nullptr;
    unsigned *d_bar = nullptr;
    size_t step_zero_words = 0;
    float *gu = nullptr;
    float *gu_split = nullptr;  // (max_batch, 2 Fl) fp32: gate/up of a split-K batched decode projection
    float *qkv_split = nullptr; // (max_batch, QKVl) fp32: QKV of a split-K batched decode projection
    float *part_split = nullptr; // (max_batch, D) fp32: O / down partial of a split-K tensor-parallel decode
    // (both accumulate with atomics and are zeroed again by the kernel that reads them, so no zeroing launch)
    float *cand_val = nullptr;  // (max_batch, 4 x lm_head tiles) argmax candidates of the batched lm_head
    int *cand_idx = nullptr;
    unsigned long long *d_trace = nullptr;  // per-phase timestamps of a profiled step
    unsigned *xch = nullptr;                // this rank's exchange buffer (tensor parallel step kernel)
    std::vector<void *> xch_peer;           // peers' exchange buffers opened through CUDA IPC
    unsigned **d_xch = nullptr;             // device array of all ranks' exchange buffers
    unsigned long long *ar_buf = nullptr;   // this rank's all-reduce inboxes (batched decode under tensor parallelism)
    unsigned long long **d_ar = nullptr;    // device array of all ranks' all-reduce inboxes
    unsigned *ar_ctr = nullptr;             // generation | CTA arrivals of the all-reduce kernel
    long long ar_cap = 0;                   // elements one all-reduce may carry
    long long ar_xoff = 0;                  // word offset of the QK-norm sums inbox ([max_batch][tp][2]) in ar_buf
    bool ar_fuse = true;                    // batched decode: all-reduce + rmsnorm and the QK sums in one kernel each
    bool prefill_sp = true;                 // tensor-parallel prefill: reduce-scatter / row-block norm / all-gather
    unsigned *d_persist = nullptr;          // barrier generation + release word, persistent
    // sampling (qw_set_sampling): temperature <= 0 keeps greedy decoding
    double samp_temperature = 0.0, samp_top_p = 1.0;
    int samp_mode = 0;
    unsigned long long *d_rng = nullptr;    // (B) java.util.Random states
    double *d_samp = nullptr;               // (B, V) probabilities
    // graph
    cudaGraphExec_t graph = nullptr;
    int launches = 0;
    // per-launch profiling (qw_profile_decode)
    bool prof_on = false;
    int prof_n = 0;
    std::vector<cudaEvent_t> prof_ev;
    std::vector<int> prof_kinds;
    std::string err;
};

namespace {

qw_status fail(qw_model *m, qw_status s, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (m) m->err = buf;
    return s;
}

#define CK(call)                                                                                        \
    do {                                                                                                \
        cudaError_t e_ = (call);                                                                        \
        if (e_ != cudaSuccess)                                                                          \
            return fail(m, e_ == cudaErrorMemoryAllocation ? QW_ERR_OOM : QW_ERR_CUDA, "%s: %s (%s:%d)", \
                        #call, cudaGetErrorString(e_), __FILE__, __LINE__);                             \
    } while (0)
#define NK(call)                                                                                         \
    do {                                                                                                 \
        ncclResult_t r_ = (call);                                                                        \
        if (r_ != ncclSuccess)                                                                           \
            return fail(m, QW_ERR_NCCL, "%s: %s (%s:%d)", #call, ncclGetErrorString(r_), __FILE__, __LINE__); \
    } while (0)
// kernel launch: counted, and bracketed by events when a profiling step is being recorded
#define LKK(kind, call)                                                          \
    do {                                                                         \
        bool prof_ = m->prof_on && m->prof_n < (int)m->prof_kinds.size();        \
        if (prof_) CK(cudaEventRecord(m->prof_ev[2 * m->prof_n], m->st));        \
        CK(call);                                                                \
        if (prof_) {                                                             \
            CK(cudaEventRecord(m->prof_ev[2 * m->prof_n + 1], m->st));           \
            m->prof_kinds[m->prof_n++] = (kind);                                 \
        }                                                                        \
        m->launches++;                                                           \
    } while (0)
#define LK(call) LKK(QW_KERNEL_OTHER, call)

template <typename T>
qw_status dalloc(qw_model *m, T **p, size_t n) {
    *p = nullptr;
    if (!n) return QW_OK;
    CK(cudaMalloc((void **)p, n * sizeof(T)));
    return QW_OK;
}
qw_status dalloc_bytes(qw_model *m, void **p, size_t n) {
    *p = nullptr;
    if (!n) return QW_OK;
    CK(cudaMalloc(p, n));
    return QW_OK;
}
#define AL(ptr, n)                                   \
    do {                                             \
        qw_status s_ = dalloc(m, &(ptr), (size_t)(n)); \
        if (s_) return s_;                           \
    } while (0)
#define ALB(ptr, n)                                        \
    do {                                                   \
        qw_status s_ = dalloc_bytes(m, (void **)&(ptr), (size_t)(n)); \
        if (s_) return s_;                                 \
    } while (0)

// ------------------------------------------------------------------------------------------
// tensor addressing: each HF key -> full shape, this rank's slice, destination
// ------------------------------------------------------------------------------------------
struct Target {
    long long full_rows = 0, full_cols = 0;  // logical full tensor (vector: rows=1)
    int r0 = 0, rows = 0, c0 = 0, cols = 0;   // slice of the full tensor this rank keeps
    void *dst = nullptr;
    bool dst_bf16 = false;
    int dst_ld = 0, dst_row0 = 0, row_map = 0;
    uint32_t tensor_id = 0;
    bool is_norm = false;  // synthetic init: ones
    uint32_t *loaded = nullptr;
    uint32_t bit = 0;
};

// returns 0 ok, -1 unknown key, -2 not used by this config (e.g. bias without has_qkv_bias)
int resolve(qw_model *m, const char *key, Target &t) {
    const qw_config &c = m->c;
    const int D = c.dim, Q = c.heads * c.head_dim, KV = c.kv_heads * c.head_dim, F = c.hidden_dim, V = c.vocab;
    const int r = m->rank;
    if (!strcmp(key, "model.embed_tokens.weight")) {
        t.full_rows = V; t.full_cols = D; t.r0 = 0; t.rows = V; t.c0 = 0; t.cols = D;
        t.dst = m->embed; t.dst_bf16 = m->bf16w; t.dst_ld = D; t.tensor_id = 0;
        t.loaded = &m->top_loaded; t.bit = 1u << K_EMBED;
        return 0;
    }
    if (!strcmp(key, "lm_head.weight")) {
        if (c.shared_weights) return -2;
        t.full_rows = V; t.full_cols = D; t.r0 = m->v0; t.rows = m->Vl; t.c0 = 0; t.cols = D;
        t.dst = m->lm; t.dst_bf16 = m->bf16w; t.dst_ld = D; t.tensor_id = 1;
        t.loaded = &m->top_loaded; t.bit = 1u << K_LMHEAD;
        return 0;
    }
    if (!strcmp(key, "model.norm.weight")) {
        t.full_rows = 1; t.full_cols = D; t.rows = 1; t.cols = D;
        t.dst = m->norm_final; t.dst_ld = D; t.tensor_id = 2; t.is_norm = true;
        t.loaded = &m->top_loaded; t.bit = 1u << K_NORM;
        return 0;
    }
    if (!strcmp(key, "rope.freq_cis")) {
        // an explicit RoPE table (seq_len, head_dim / 2, 2) = (cos, sin), as Llama2 checkpoints carry
        // (Llama2Weights.java freqCis); replaces the one computed from rope_theta.  Optional.
        t.full_rows = 1; t.full_cols = (long long)c.seq_len * c.head_dim; t.rows = 1; t.cols = c.seq_len * c.head_dim;
        t.dst = m->freq; t.dst_ld = t.cols; t.tensor_id = 3;
        t.loaded = &m->top_loaded; t.bit = 1u << K_FREQ;
        return 0;
    }
    int l = -1, n = 0;
    char rest[128];
    if (sscanf(key, "model.layers.%d.%127s%n", &l, rest, &n) != 2 || l < 0 || l >= c.layers) return -1;
    int kind = -1;
    for (int k = 0; k < K_NUM_LAYER_KINDS; k++)
        if (!strcmp(rest, kLayerNames[k])) kind = k;
    if (kind < 0) return -1;
    if ((kind == K_BQ || kind == K_BK || kind == K_BV) && !c.has_qkv_bias) return -2;
    if ((kind == K_QN || kind == K_KN) && c.qk_norm == QW_QKNORM_NONE) return -2;
    Layer &Ly = m->L[l];
    t.tensor_id = 16u + (uint32_t)l * 16u + (uint32_t)kind;
    t.loaded = &Ly.loaded;
    t.bit = 1u << kind;
    const int Ql = m->Ql, KVl = m->KVl, Fl = m->Fl;
    switch (kind) {
        case K_RMS_ATT: case K_RMS_FFN:
            t.full_rows = 1; t.full_cols = D; t.rows = 1; t.cols = D; t.dst_ld = D; t.is_norm = true;
            t.dst = kind == K_RMS_ATT ? Ly.rms_att : Ly.rms_ffn;
            break;
        case K_WQ: case K_WK: case K_WV: {
            int full = kind == K_WQ ? Q : KV, loc = kind == K_WQ ? Ql : KVl;
            t.full_rows = full; t.full_cols = D; t.r0 = r * loc; t.rows = loc; t.cols = D;
            t.dst = Ly.w_qkv; t.dst_bf16 = m->bf16w; t.dst_ld = D;
            t.dst_row0 = kind == K_WQ ? 0 : (kind == K_WK ? Ql : Ql + KVl);
            break;
        }
        case K_BQ: case K_BK: case K_BV: {
            int full = kind == K_BQ ? Q : KV, loc = kind == K_BQ ? Ql : KVl;
            // vectors are treated as (full, 1) column tensors so that the row slice applies
            t.full_rows = full; t.full_cols = 1; t.r0 = r * loc; t.rows = loc; t.cols = 1;
            t.dst = Ly.b_qkv; t.dst_ld = 1; t.dst_row0 = kind == K_BQ ? 0 : (kind == K_BK ? Ql : Ql + KVl);
            break;
        }
        case K_QN: case K_KN: {
            int full = kind == K_QN ? Q : KV, loc = kind == K_QN ? Ql : KVl;
            t.full_rows = full; t.full_cols = 1; t.r0 = r * loc; t.rows = loc; t.cols = 1;
            t.dst = kind == K_QN ? Ly.qn : Ly.kn; t.dst_ld = 1; t.is_norm = true;
            break;
        }
        case K_WO:
            t.full_rows = D; t.full_cols = Q; t.r0 = 0; t.rows = D; t.c0 = r * Ql; t.cols = Ql;
            t.dst = Ly.w_o; t.dst_bf16 = m->bf16w; t.dst_ld = Ql;
            break;
        case K_W1: case K_W3:
            t.full_rows = F; t.full_cols = D; t.r0 = r * Fl; t.rows = Fl; t.cols = D;
            t.dst = Ly.w_gu; t.dst_bf16 = m->bf16w; t.dst_ld = D; t.row_map = kind == K_W1 ? 1 : 2;
            break;
        case K_W2:
            t.full_rows = D; t.full_cols = F; t.r0 = 0; t.rows = D; t.c0 = r * Fl; t.cols = Fl;
            t.dst = Ly.w_down; t.dst_bf16 = m->bf16w; t.dst_ld = Fl;
            break;
    }
    return 0;
}

uint32_t required_layer_bits(const qw_config &c) {
    uint32_t bits = 0;
    for (int k = 0; k < K_NUM_LAYER_KINDS; k++) {
        if ((k == K_BQ || k == K_BK || k == K_BV) && !c.has_qkv_bias) continue;
        if ((k == K_QN || k == K_KN) && c.qk_norm == QW_QKNORM_NONE) continue;
        bits |= 1u << k;
    }
    return bits;
}

qw_status place(qw_model *m, const Target &t, const void *src, int src_dtype, int src_ld, bool synth, uint64_t seed,
                float stdv) {
    PlaceArgs p{};
    p.dst = t.dst; p.dst_bf16 = t.dst_bf16; p.dst_ld = t.dst_ld; p.dst_row0 = t.dst_row0; p.row_map = t.row_map;
    p.rows = t.rows; p.cols = t.cols;
    p.src = src; p.src_dtype = src_dtype; p.src_ld = src_ld;
    p.synth = synth; p.constant_one = synth && t.is_norm; p.seed = seed; p.tensor_id = t.tensor_id;
    // Irwin-Hall(4) of 16-bit uniforms: variance 4 * (65536^2 - 1) / 12
    p.scale = (float)(stdv / sqrt(4.0 * (65536.0 * 65536.0 - 1.0) / 12.0));
    p.src_row0 = t.r0; p.src_col0 = t.c0; p.full_cols = t.full_cols;
    CK(place_launch(p, m->st));
    return QW_OK;
}

// ------------------------------------------------------------------------------------------
// paged KV
// ------------------------------------------------------------------------------------------
qw_status reserve_pages(qw_model *m, int slot, int npos) {
    if (slot < 0 || slot >= m->B) return fail(m, QW_ERR_ARG, "slot %d out of range [0,%d)", slot, m->B);
    if (npos > m->c.seq_len) return fail(m, QW_ERR_SHAPE, "position %d beyond seq_len %d", npos, m->c.seq_len);
    int need = (npos + m->page_size - 1) / m->page_size;
    auto &sp = m->slot_pages[slot];
    int have = (int)sp.size();
    if (need <= have) return QW_OK;
    if ((int)m->free_pages.size() < need - have)
        return fail(m, QW_ERR_OOM, "KV cache exhausted: slot %d needs %d more pages, %zu free", slot, need - have,
                    m->free_pages.size());
    for (int i = have; i < need; i++) {
        int pg = m->free_pages.back();
        m->free_pages.pop_back();
        sp.push_back(pg);
        m->h_page_table[(size_t)slot * m->max_pages + i] = pg;
    }
    CK(cudaMemcpy(m->d_page_table + (size_t)slot * m->max_pages + have,
                  m->h_page_table.data() + (size_t)slot * m->max_pages + have, sizeof(int) * (need - have),
                  cudaMemcpyHostToDevice));
    return QW_OK;
}

void release_slot(qw_model *m, int slot) {
    auto &sp = m->slot_pages[slot];
    for (int pg : sp) m->free_pages.push_back(pg);
    sp.clear();
}

// ------------------------------------------------------------------------------------------
// the decode step (batch <= kGemvMaxB per pass) -- all pointers device-resident
// ------------------------------------------------------------------------------------------
int choose_nsplit(qw_model *m, int B) {
    int per = B * m->Hkvl;
    int ns = (2 * m->num_sms + per - 1) / per;
    int cap = (m->c.seq_len + 63) / 64;
    ns = std::min(ns, cap);
    ns = std::min(ns, m->maxsplit);
    return std::max(ns, 1);
}

// context splits of the tensor-core decode attention: about four CTAs per SM, at most one split per
// 64-key tile of the longest possible context
// Context splits of flash decoding.  B x Hkv x ns CTAs run 2 per SM (98 KB of shared memory each); a CTA's time
// is about its share of the context, 1 / ns, so ns minimises waves(ns) / ns plus a small merge cost per split:
// whole waves, not a half-empty last one (B 64, Hkv 8: 4 splits = 6.9 waves rather than 2 splits = 3.5 waves).
int choose_flash_split(qw_model *m, int B) {
    const int per = B * m->Hkvl;
    const int resident = 2 * m->num_sms;
    const int ntiles = (m->c.seq_len + 63) / 64;  // 64-key tiles at the longest context
    const int hi = std::max(1, std::min(ntiles, m->maxsplit));
    // QW_FLASH_FIXED overrides the fixed cost (a negative value restores the older waves / splits model)
    static const double fixed = [] {
        const char *e = getenv("QW_FLASH_FIXED");
        return e ? atof(e) : 4.0;
    }();
    int best_ns = 1;
    double best = 1e30;
    for (int ns = 1; ns <= hi; ns++) {
        const double waves = (double)(((long long)per * ns + resident - 1) / resident);
        double cost;
        if (fixed >= 0) {
            // waves x (tiles per CTA + a CTA's fixed cost in tiles: set-up, first-load latency, split merge)
            cost = waves * ((ntiles + ns - 1) / ns + fixed);
        } else {
            cost = waves / ns + 0.005 * ns;
        }
        if (cost < best - 1e-9) { best = cost; best_ns = ns; }
    }
    return best_ns;
}

qw_status allreduce(qw_model *m, float *buf, size_t n) {
    if (m->ar_buf && (long long)n <= m->ar_cap) {
        // decode-sized: the two-shot flag-in-data kernel over NVLink (qw_allreduce.cu)
        ArArgs a{};
        a.x = buf; a.n = (long long)n; a.tp = m->tp; a.rank = m->rank; a.peers = m->d_ar;
        a.gather_off = (long long)m->tp * (((long long)n + m->tp - 1) / m->tp);
        a.gen = m->ar_ctr; a.done = m->ar_ctr + 1; a.err = m->pf.d_err;
        LK(allreduce_ll_launch(a, m->num_sms, m->st));
        return QW_OK;
    }
    NK(ncclAllReduce(buf, buf, n, ncclFloat, ncclSum, m->comm, m->st));
    return QW_OK;
}

// Tensor-parallel tail: all-gather every rank's (value, index) winner and its logits shard.
qw_status tp_merge_argmax(qw_model *m, int B, float *logits_out_dev, int *argmax_dev, int *next_tokens, int *positions,
                          int advance, int *hist, int hist_ld) {
    NK(ncclAllGather(m->am_val, m->am_val_all, B, ncclFloat, m->comm, m->st));
    NK(ncclAllGather(m->am_idx, m->am_idx_all, B, ncclInt32, m->comm, m->st));
    LK(argmax_merge_launch(m->am_val_all, m->am_idx_all, m->tp, B, argmax_dev, next_tokens, positions, advance, hist,
                           hist_ld, m->st));
    if (logits_out_dev) {
        NK(ncclAllGather(m->logits, m->logits_all, (size_t)B * m->Vl, ncclFloat, m->comm, m->st));
        // logits_all is [rank][b][Vl] -> logits_out_dev [b][V]
        for (int r = 0; r < m->tp; r++)
            CK(cudaMemcpy2DAsync(logits_out_dev + (size_t)r * m->Vl, sizeof(float) * m->c.vocab,
                                 m->logits_all + (size_t)r * B * m->Vl, sizeof(float) * m->Vl, sizeof(float) * m->Vl,
                                 B, cudaMemcpyDeviceToDevice, m->st));
    }
    return QW_OK;
}

// Final rmsnorm + lm_head + greedy argmax for B <= kGemvMaxB rows x (row b at xin + b * ld_in, plus an
// optional all-reduced partial), merged across tensor-parallel ranks.
qw_status lm_head_gemv(qw_model *m, const float *xin, int ld_in, const float *pending, int ld_part, int B,
                       float *logits_out_dev, int *argmax_dev, int *next_tokens, int *positions, int advance, int *hist,
                       int hist_ld) {
    const qw_config &c = m->c;
    const int D = m->D;
    const bool tpm = m->tp > 1;
    GemvArgs g{};
    g.W = m->lm; g.N = m->Vl; g.K = D; g.B = B; g.xin = xin; g.ld_in = ld_in;
    if (pending) { g.part = pending; g.ld_part = ld_part; }
    g.norm_w = m->norm_final; g.eps = (float)c.eps;
    g.out = tpm ? m->logits : logits_out_dev; g.ld_out = m->Vl;
    if (tpm && !logits_out_dev) g.out = nullptr;
    g.part_val = m->am_pval; g.part_idx = m->am_pidx; g.counter = m->am_counter; g.idx_offset = m->v0;
    if (!tpm) {
        g.argmax_out = argmax_dev; g.next_tokens = next_tokens; g.positions = positions; g.advance = advance;
        g.hist = hist; g.hist_ld = hist_ld;
    } else {
        g.argmax_out = m->am_idx; g.argmax_val = m->am_val;
    }
    LKK(QW_KERNEL_LM_HEAD, gemv_launch(g, EPI_ARGMAX, m->bf16w, m->num_sms, m->st));
    if (tpm) return tp_merge_argmax(m, B, logits_out_dev, argmax_dev, next_tokens, positions, advance, hist, hist_ld);
    return QW_OK;
}

// One forward for B <= 4 rows.  tokens: device token ids (or null when x_in given: fp32 (B, D)).
qw_status decode_pass(qw_model *m, const int *tokens, const float *x_in, const int *slots, int *positions, int B,
                      float *logits_out_dev, int *argmax_dev, int *next_tokens, int advance, int *hist, int hist_ld) {
    const qw_config &c = m->c;
    const int D = m->D, d = c.head_dim;
    const bool tpm = m->tp > 1;
    float *xcur = m->xa, *xalt = m->xb;
    const float *pending = nullptr;  // all-reduced partial to be added to xcur (tp > 1)
    if (B == 1 && tokens && !x_in && m->use_step) {
        StepArgs sa = m->step;
        sa.tokens = next_tokens ? next_tokens : const_cast<int *>(tokens);
        sa.positions = positions; sa.slots = slots; sa.advance = advance; sa.hist = hist;
        // under tensor parallelism every rank writes its vocabulary shard, gathered below
        sa.argmax_out = argmax_dev; sa.logits = tpm && logits_out_dev ? m->logits : logits_out_dev;
        sa.trace = m->prof_on ? m->d_trace : nullptr;
        CK(cudaMemsetAsync(sa.bar, 0, sizeof(unsigned) * m->step_zero_words, m->st));
        LKK(QW_KERNEL_STEP, step_launch(sa, m->bf16kv, m->num_sms, m->st));
        if (tpm && logits_out_dev) {
            NK(ncclAllGather(m->logits, m->logits_all, (size_t)m->Vl, ncclFloat, m->comm, m->st));
            CK(cudaMemcpyAsync(logits_out_dev, m->logits_all, sizeof(float) * m->c.vocab, cudaMemcpyDeviceToDevice,
                               m->st));
        }
        return QW_OK;
    }
    int nsplit = choose_nsplit(m, B);
    const void *W_embed = m->embed;
    if (x_in) {
        CK(cudaMemcpyAsync(xcur, x_in, sizeof(float) * B * D, cudaMemcpyDeviceToDevice, m->st));
    }
    for (int l = 0; l < c.layers; l++) {
        Layer &Ly = m->L[l];
        // ---- rmsnorm + fused QKV projection (+bias) ----
        GemvArgs g{};
        g.W = Ly.w_qkv; g.N = m->QKVl; g.K = D; g.B = B;
        if (l == 0 && !x_in) { g.embed = W_embed; g.tokens = tokens; g.xsave = xcur; g.ld_xsave = D; }
        else { g.xin = xcur; g.ld_in = D; }
        if (pending) { g.part = pending; g.ld_part = D; g.xsave = xalt; g.ld_xsave = D; }
        g.norm_w = Ly.rms_att; g.eps = (float)c.eps;
        g.out = m->qkv; g.ld_out = m->QKVl; g.bias = Ly.b_qkv;
        LKK(QW_KERNEL_QKV, gemv_launch(g, EPI_STORE, m->bf16w, m->num_sms, m->st));
        if (pending) { std::swap(xcur, xalt); pending = nullptr; }
        // ---- QK-norm + RoPE + KV write + attention ----
        const float *qk_ss = nullptr;
        if (tpm && c.qk_norm == QW_QKNORM_VECTOR) {
            LK(qk_sumsq_launch(m->qkv, m->QKVl, m->Ql, m->KVl, B, m->qk_ss, m->st));
            qw_status s = allreduce(m, m->qk_ss, (size_t)B * 2);
            if (s) return s;
            qk_ss = m->qk_ss;
        }
        AttnArgs a{};
        a.qkv = m->qkv; a.ld_qkv = m->QKVl; a.qn = Ly.qn; a.kn = Ly.kn; a.qk_mode = c.qk_norm; a.qk_ss = qk_ss;
        a.q_total = c.heads * d; a.kv_total = c.kv_heads * d;
        a.freq = m->freq;
        a.kcache = (char *)m->kpool + (size_t)l * m->layer_kv_elems * m->kvsz;
        a.vcache = (char *)m->vpool + (size_t)l * m->layer_kv_elems * m->kvsz;
        a.page_table = m->d_page_table; a.max_pages = m->max_pages; a.slots = slots; a.positions = positions;
        a.H = m->Hl; a.Hkv = m->Hkvl; a.d = d; a.page_size = m->page_size; a.log2_page = m->log2_page;
        a.nsplit = nsplit; a.scale = (float)(1.0 / sqrt((double)d));
        a.part_o = m->part_o; a.part_ml = m->part_ml; a.counters = m->counters;
        a.out = m->attn; a.ld_out = m->Ql;
        LKK(QW_KERNEL_ATTN, attn_decode_launch(a, B, m->bf16kv, m->st));
        // ---- O projection + residual ----
        g = GemvArgs{};
        g.W = Ly.w_o; g.N = D; g.K = m->Ql; g.B = B; g.xin = m->attn; g.ld_in = m->Ql;
        if (tpm) { g.out = m->part; g.ld_out = D; }
        else { g.out = xalt; g.ld_out = D; g.resid = xcur; g.ld_resid = D; }
        LKK(QW_KERNEL_O, gemv_launch(g, EPI_RESID, m->bf16w, m->num_sms, m->st));
        if (tpm) {
            qw_status s = allreduce(m, m->part, (size_t)B * D);
            if (s) return s;
            pending = m->part;
        } else std::swap(xcur, xalt);
        // ---- rmsnorm + gate/up + SwiGLU ----
        g = GemvArgs{};
        g.W = Ly.w_gu; g.N = 2 * m->Fl; g.K = D; g.B = B; g.xin = xcur; g.ld_in = D;
        if (pending) { g.part = pending; g.ld_part = D; g.xsave = xalt; g.ld_xsave = D; }
        g.norm_w = Ly.rms_ffn; g.eps = (float)c.eps;
        g.out = m->hbuf; g.ld_out = m->Fl;
        LKK(QW_KERNEL_GATE_UP, gemv_launch(g, EPI_SWIGLU, m->bf16w, m->num_sms, m->st));
        if (pending) { std::swap(xcur, xalt); pending = nullptr; }
        // ---- down projection + residual ----
        g = GemvArgs{};
        g.W = Ly.w_down; g.N = D; g.K = m->Fl; g.B = B; g.xin = m->hbuf; g.ld_in = m->Fl;
        if (tpm) { g.out = m->part; g.ld_out = D; }
        else { g.out = xalt; g.ld_out = D; g.resid = xcur; g.ld_resid = D; }
        LKK(QW_KERNEL_DOWN, gemv_launch(g, EPI_RESID, m->bf16w, m->num_sms, m->st));
        if (tpm) {
            qw_status s = allreduce(m, m->part, (size_t)B * D);
            if (s) return s;
            pending = m->part;
        } else std::swap(xcur, xalt);
    }
    return lm_head_gemv(m, xcur, D, pending, D, B, logits_out_dev, argmax_dev, next_tokens, positions, advance, hist,
                        hist_ld);
}

// ------------------------------------------------------------------------------------------
// the batched step on the tensor cores: prefill chunks and decode batches above kGemvMaxB
// ------------------------------------------------------------------------------------------
qw_status tc_gemm(qw_model *m, int kind, const void *W, const void *X, int M, int T, int K, int epi, void *out,
                  int ld_out, const float *resid, const float *bias, bool allow_split) {
    TcArgs a{};
    const int bn = tc_pick_bn(T);
    a.M = M; a.T = T; a.K = K;
    a.ksplit = allow_split ? tc_pick_ksplit(M, T, K, bn, m->num_sms) : 1;
    a.out = out; a.ld_out = ld_out; a.resid = resid; a.ld_resid = ld_out; a.bias = bias; a.err = m->pf.d_err;
    // a split STORE accumulates with atomics into a buffer its consumer keeps zeroed (qkv_split, gu_split)
    LKK(kind, tc_gemm_launch(W, X, a, epi, bn, m->num_sms, m->st));
    return QW_OK;
}

#define TRY(call)                  \
    do {                           \
        qw_status s_ = (call);     \
        if (s_) return s_;         \
    } while (0)

// All layers for T token rows (row r: token tokens[r] or hidden x_in row r, at slot row_slot[r] and
// position row_pos[r]).  prefill: the rows are nseq sequences of L consecutive positions from p0
// (flash attention); otherwise T single-token sequences (paged decode attention).  Leaves the
// residual stream in m->xa and, under tensor parallelism, the last all-reduced partial in *pending.
qw_status tc_layers(qw_model *m, int T, const int *tokens, const float *x_in, const int *row_slot, const int *row_pos,
                    bool prefill, int nseq, int p0, int L, const int *seq_slots, const float **pending_out,
                    bool *final_normed = nullptr, bool *seq_par = nullptr) {
    const qw_config &c = m->c;
    PrefillBuffers &pf = m->pf;
    const int D = m->D, d = c.head_dim;
    const bool tpm = m->tp > 1;
    // tensor-parallel decode: each all-reduce fused with the residual update and the next rmsnorm (qw_ar_norm_kernel),
    // the QK-norm sums exchanged inside qkv_post; the last layer's down all-reduce applies the final norm
    const bool fuse = tpm && !prefill && m->ar_fuse && m->ar_buf && (long long)T * D <= m->ar_cap &&
                      T <= m->num_sms && m->tp <= 8 && D % (4 * m->tp) == 0;
    if (final_normed) *final_normed = fuse;
    // tensor-parallel prefill, sequence-parallel between the projections: the O / down partials are reduce-scattered
    // (each rank gets its block of T / tp rows summed), the residual update and rmsnorm run on that block only, and
    // the normalised bf16 rows are all-gathered as the next projection's operand: 3/4 of an fp32 all-reduce's bytes
    // and 1/tp of the row work.  The residual stream is then current only in this rank's row block.
    const bool sp = tpm && prefill && m->prefill_sp && T % m->tp == 0;
    if (seq_par) *seq_par = sp;
    const int Tl = sp ? T / m->tp : T, rb = sp ? m->rank * Tl : 0;  // this rank's row block
    auto sp_norm = [&](const float *part, const float *w, const int *tok) -> qw_status {
        NormRowsArgs nb{};
        nb.x = m->xa + (size_t)rb * D; nb.ld_x = D; nb.part = const_cast<float *>(part); nb.ld_part = D;
        if (tok) { nb.embed = (const __nv_bfloat16 *)m->embed; nb.tokens = tok + rb; }
        nb.w = w; nb.eps = (float)c.eps; nb.out = pf.act + (size_t)rb * D; nb.ld_out = D; nb.K = D;
        LK(norm_rows_launch(nb, Tl, m->st));
        NK(ncclAllGather(pf.act + (size_t)rb * D, pf.act, (size_t)Tl * D, ncclBfloat16, m->comm, m->st));
        return QW_OK;
    };
    auto sp_reduce = [&](float *part) -> qw_status {
        NK(ncclReduceScatter(part, part + (size_t)rb * D, (size_t)Tl * D, ncclFloat, ncclSum, m->comm, m->st));
        return QW_OK;
    };
    const float *sp_pending = nullptr;  // this rank's block of the last reduce-scattered partial
    auto ar_norm = [&](float *part, const float *w) -> qw_status {
        ArNormArgs an{};
        an.part = part; an.ld_part = D; an.zero_part = part == m->part_split;
        an.x = m->xa; an.w = w; an.eps = (float)c.eps; an.out = pf.act; an.ld_out = D; an.D = D; an.rows = T;
        an.tp = m->tp; an.rank = m->rank; an.peers = m->d_ar; an.gen = m->ar_ctr; an.done = m->ar_ctr + 1;
        an.err = pf.d_err;
        LK(ar_norm_launch(an, m->num_sms, m->st));
        return QW_OK;
    };
    float *x = m->xa;
    const float *pending = nullptr;
    if (x_in) CK(cudaMemcpyAsync(x, x_in, sizeof(float) * (size_t)T * D, cudaMemcpyDeviceToDevice, m->st));
    for (int l = 0; l < c.layers; l++) {
        Layer &Ly = m->L[l];
        // ---- residual update + rmsnorm -> bf16 rows (fused: done by the previous layer's last all-reduce) ----
        NormRowsArgs na{};
        if (sp) {
            TRY(sp_norm(sp_pending, Ly.rms_att, l == 0 ? tokens : nullptr));
            sp_pending = nullptr;
        } else if (!fuse || l == 0) {
            na.x = x; na.ld_x = D; na.part = const_cast<float *>(pending); na.ld_part = D; na.zero_part = pending == m->part_split;
            if (l == 0 && !x_in) { na.embed = (const __nv_bfloat16 *)m->embed; na.tokens = tokens; }
            na.w = Ly.rms_att; na.eps = (float)c.eps; na.out = pf.act; na.ld_out = D; na.K = D;
            LK(norm_rows_launch(na, T, m->st));
        }
        pending = nullptr;
        // ---- fused QKV projection ----
        // split K (skinny decode shapes): atomics into qkv_split, which qkv_post zeroes again after reading it
        const bool qkv_sp = T <= m->B && tc_pick_ksplit(m->QKVl, T, D, tc_pick_bn(T), m->num_sms) > 1;
        float *qkv = qkv_sp ? m->qkv_split : m->qkv;
        TRY(tc_gemm(m, QW_KERNEL_QKV, Ly.w_qkv, pf.act, m->QKVl, T, D, TC_STORE, qkv, m->QKVl, nullptr, Ly.b_qkv,
                    qkv_sp));
        const float *qk_ss = nullptr;
        if (tpm && c.qk_norm == QW_QKNORM_VECTOR && !fuse) {
            LK(qk_sumsq_launch(qkv, m->QKVl, m->Ql, m->KVl, T, pf.row_ss, m->st));
            TRY(allreduce(m, pf.row_ss, (size_t)T * 2));
            qk_ss = pf.row_ss;
        }
        void *kc = (char *)m->kpool + (size_t)l * m->layer_kv_elems * m->kvsz;
        void *vc = (char *)m->vpool + (size_t)l * m->layer_kv_elems * m->kvsz;
        {
            QkvPostArgs qa{};
            qa.qkv = qkv; qa.zero_qkv = qkv_sp; qa.ld_qkv = m->QKVl; qa.qn = Ly.qn; qa.kn = Ly.kn; qa.qk_mode = c.qk_norm; qa.qk_ss = qk_ss;
            qa.q_total = c.heads * d; qa.kv_total = c.kv_heads * d; qa.freq = m->freq;
            qa.slots = row_slot; qa.positions = row_pos; qa.page_table = m->d_page_table; qa.max_pages = m->max_pages;
            qa.page_size = m->page_size; qa.log2_page = m->log2_page; qa.kcache = kc; qa.vcache = vc;
            qa.H = m->Hl; qa.Hkv = m->Hkvl; qa.d = d; qa.q_out = pf.q; qa.ld_q = m->Ql;
            if (fuse && c.qk_norm == QW_QKNORM_VECTOR) {
                qa.xpeers = m->d_ar; qa.xoff = m->ar_xoff; qa.tp = m->tp; qa.rank = m->rank;
                qa.gen = m->ar_ctr; qa.done = m->ar_ctr + 1; qa.err = pf.d_err;
            }
            LK(qkv_post_launch(qa, T, m->bf16kv, m->st));
        }
        if (prefill) {
            FlashArgs fa{};
            fa.q = pf.q; fa.ld_q = m->Ql; fa.kcache = kc; fa.vcache = vc; fa.page_table = m->d_page_table;
            fa.max_pages = m->max_pages; fa.page_size = m->page_size; fa.log2_page = m->log2_page;
            fa.seq_slots = seq_slots; fa.p0 = p0; fa.L = L; fa.H = m->Hl; fa.Hkv = m->Hkvl; fa.d = d;
            fa.scale = (float)(1.0 / sqrt((double)d)); fa.out = pf.act; fa.ld_out = m->Ql;
            fa.num_pages = m->num_pages; fa.err = pf.d_err;
            if (d == 128 && m->tc_attn && !(m->Hl / m->Hkvl & (m->Hl / m->Hkvl - 1))) LKK(QW_KERNEL_ATTN, flash_prefill_tc_launch(fa, nseq, m->st));
            else LKK(QW_KERNEL_ATTN, flash_prefill_launch(fa, nseq, m->st));
        } else {
            FlashDecodeArgs fd{};
            fd.q = pf.q; fd.ld_q = m->Ql; fd.kcache = kc; fd.vcache = vc; fd.page_table = m->d_page_table;
            fd.max_pages = m->max_pages; fd.page_size = m->page_size; fd.log2_page = m->log2_page;
            fd.slots = row_slot; fd.positions = row_pos; fd.H = m->Hl; fd.Hkv = m->Hkvl; fd.d = d;
            fd.nsplit = choose_flash_split(m, T); fd.scale = (float)(1.0 / sqrt((double)d));
            fd.part_o = m->part_o; fd.part_ml = m->part_ml; fd.counters = m->counters;
            fd.out = pf.act; fd.ld_out = m->Ql; fd.num_pages = m->num_pages; fd.err = pf.d_err;
            LKK(QW_KERNEL_ATTN, flash_decode_launch(fd, T, m->st));
        }
        // ---- O projection (+ residual) ----
        if (tpm) {
            // decode: split K with atomics into part_split, which the next rmsnorm zeroes again after reading it
            const bool ksp = !prefill && T <= m->B;
            float *pb = ksp ? m->part_split : m->part;
            TRY(tc_gemm(m, QW_KERNEL_O, Ly.w_o, pf.act, D, T, m->Ql, TC_STORE, pb, D, nullptr, nullptr, ksp));
            if (fuse) {
                TRY(ar_norm(pb, Ly.rms_ffn));
            } else if (sp) {
                TRY(sp_reduce(pb));
                TRY(sp_norm(pb + (size_t)rb * D, Ly.rms_ffn, nullptr));
            } else {
                TRY(allreduce(m, pb, (size_t)T * D));
                pending = pb;
            }
        } else {
            TRY(tc_gemm(m, QW_KERNEL_O, Ly.w_o, pf.act, D, T, m->Ql, TC_RESID, x, D, x, nullptr, true));
        }
        // ---- residual update + rmsnorm ----
        if (!fuse && !sp) {
            na = NormRowsArgs{};
            na.x = x; na.ld_x = D; na.part = const_cast<float *>(pending); na.ld_part = D; na.zero_part = pending == m->part_split;
            na.w = Ly.rms_ffn; na.eps = (float)c.eps; na.out = pf.act; na.ld_out = D; na.K = D;
            LK(norm_rows_launch(na, T, m->st));
        }
        pending = nullptr;
        // ---- gate/up + SwiGLU, down (+ residual) ----
        if (!prefill && T <= m->B && m->gu_split && tc_pick_ksplit(2 * m->Fl, T, D, tc_pick_bn(T), m->num_sms) > 1) {
            // too few output tiles to fill the GPU: split K into an fp32 buffer, then SwiGLU row by row (the
            // SwiGLU epilogue needs whole sums)
            TRY(tc_gemm(m, QW_KERNEL_GATE_UP, Ly.w_gu, pf.act, 2 * m->Fl, T, D, TC_STORE, m->gu_split, 2 * m->Fl, nullptr,
                        nullptr, true));
            LKK(QW_KERNEL_GATE_UP, swiglu_rows_launch(m->gu_split, T, m->Fl, pf.h, m->st));
        } else {
            TRY(tc_gemm(m, QW_KERNEL_GATE_UP, Ly.w_gu, pf.act, 2 * m->Fl, T, D, TC_SWIGLU, pf.h, m->Fl, nullptr, nullptr,
                        false));
        }
        if (tpm) {
            // decode: split K with atomics into part_split, which the next rmsnorm zeroes again after reading it
            const bool ksp = !prefill && T <= m->B;
            float *pb = ksp ? m->part_split : m->part;
            TRY(tc_gemm(m, QW_KERNEL_DOWN, Ly.w_down, pf.h, D, T, m->Fl, TC_STORE, pb, D, nullptr, nullptr, ksp));
            if (fuse) {
                TRY(ar_norm(pb, l + 1 < c.layers ? m->L[l + 1].rms_att : m->norm_final));
            } else if (sp) {
                TRY(sp_reduce(pb));
                sp_pending = pb + (size_t)rb * D;
            } else {
                TRY(allreduce(m, pb, (size_t)T * D));
                pending = pb;
            }
        } else {
            TRY(tc_gemm(m, QW_KERNEL_DOWN, Ly.w_down, pf.h, D, T, m->Fl, TC_RESID, x, D, x, nullptr, true));
        }
    }
    *pending_out = sp ? sp_pending : pending;
    return QW_OK;
}

// Decode step for B > kGemvMaxB sequences: batched layers, then rmsnorm + lm_head GEMM + row argmax.
qw_status tc_decode(qw_model *m, int *tokens, const float *x_in, const int *slots, int *positions, int B,
                    float *logits_out_dev, int *argmax_dev, int advance, int *hist, int hist_ld) {
    const float *pending = nullptr;
    bool normed = false;
    TRY(tc_layers(m, B, tokens, x_in, slots, positions, false, 0, 0, 1, nullptr, &pending, &normed));
    const bool tpm = m->tp > 1;
    if (!normed) {
        NormRowsArgs na{};
        na.x = m->xa; na.ld_x = m->D; na.part = const_cast<float *>(pending); na.ld_part = m->D; na.zero_part = pending == m->part_split;
        na.w = m->norm_final; na.eps = (float)m->c.eps; na.out = m->pf.act; na.ld_out = m->D; na.K = m->D;
        LK(norm_rows_launch(na, B, m->st));
    }
    // lm_head with the argmax candidates of every 32 vocabulary rows in its epilogue; logits only when asked for
    float *lg = logits_out_dev ? (tpm ? m->logits : logits_out_dev) : nullptr;
    const int ncand = (m->Vl + 127) / 128 * 4;
    {
        TcArgs a{};
        a.M = m->Vl; a.T = B; a.K = m->D; a.ksplit = 1;
        a.out = lg; a.ld_out = m->Vl; a.err = m->pf.d_err;
        a.cand_val = m->cand_val; a.cand_idx = m->cand_idx; a.ncand = ncand;
        LKK(QW_KERNEL_LM_HEAD, tc_gemm_launch(m->lm, m->pf.act, a, TC_ARGMAX, tc_pick_bn(B), m->num_sms, m->st));
    }
    RowsArgmaxArgs ra{};
    ra.cand_val = m->cand_val; ra.cand_idx = m->cand_idx; ra.ld = ncand; ra.n = ncand; ra.idx_offset = m->v0;
    if (!tpm) {
        ra.argmax_out = argmax_dev; ra.next_tokens = tokens; ra.positions = positions; ra.advance = advance;
        ra.hist = hist; ra.hist_ld = hist_ld;
    } else {
        ra.argmax_out = m->am_idx; ra.argmax_val = m->am_val;
    }
    LKK(QW_KERNEL_LM_HEAD, rows_argmax_launch(ra, B, m->st));
    if (tpm) return tp_merge_argmax(m, B, logits_out_dev, argmax_dev, tokens, positions, advance, hist, hist_ld);
    return QW_OK;
}

// full device step for any B (chunks of kGemvMaxB rows through the GEMV path)
qw_status device_step(qw_model *m, int *tokens, const float *x_in, const int *slots, int *positions, int B,
                      float *logits_dev, int *argmax_dev, int advance, int *hist, int hist_ld) {
    if (!m->finalized) return fail(m, QW_ERR_STATE, "weights not finalized");
    if (B < 1 || B > m->B) return fail(m, QW_ERR_SHAPE, "batch %d outside [1,%d]", B, m->B);
    m->launches = 0;
    if (B > kGemvMaxB && m->pf.tc)
        return tc_decode(m, tokens, x_in, slots ? slots : m->d_slots, positions, B, logits_dev, argmax_dev, advance,
                         hist, hist_ld);
    for (int b0 = 0; b0 < B; b0 += kGemvMaxB) {
        int nb = std::min(kGemvMaxB, B - b0);
        const int *sl = slots ? slots + b0 : nullptr;
        if (!slots) {
            // default slots 0..B-1: pass an explicit slice of the identity table
            sl = m->d_slots + b0;
        }
        qw_status s = decode_pass(m, tokens ? tokens + b0 : nullptr, x_in ? x_in + (size_t)b0 * m->D : nullptr, sl,
                                  positions + b0, nb, logits_dev ? logits_dev + (size_t)b0 * m->c.vocab : nullptr,
                                  argmax_dev ? argmax_dev + b0 : nullptr, tokens ? tokens + b0 : nullptr, advance,
                                  hist ? hist + (size_t)b0 * hist_ld : nullptr, hist_ld);
        if (s) return s;
    }
    return QW_OK;
}

qw_status check_positions(qw_model *m, const int32_t *slots, const int32_t *positions, int batch) {
    for (int b = 0; b < batch; b++) {
        int s = slots ? slots[b] : b;
        if (s < 0 || s >= m->B) return fail(m, QW_ERR_ARG, "slot %d out of range", s);
        for (int b2 = 0; b2 < b; b2++)
            if ((slots ? slots[b2] : b2) == s) return fail(m, QW_ERR_ARG, "slot %d used twice in one batch", s);
        if (positions[b] < 0 || positions[b] >= m->c.seq_len)
            return fail(m, QW_ERR_SHAPE, "position %d outside [0,%d)", positions[b], m->c.seq_len);
        qw_status st = reserve_pages(m, s, positions[b] + 1);
        if (st) return st;
    }
    return QW_OK;
}

// host-facing step: stage small int arrays through pinned memory
qw_status host_step(qw_model *m, const int32_t *tokens, const float *x_in, const int32_t *slots,
                    const int32_t *positions, int batch, float *logits_out, int32_t *argmax_out) {
    if (!m->finalized) return fail(m, QW_ERR_STATE, "weights not finalized");
    if (!positions || (!tokens && !x_in)) return fail(m, QW_ERR_ARG, "null tokens/positions");
    if (batch < 1 || batch > m->B) return fail(m, QW_ERR_SHAPE, "batch %d outside [1,%d]", batch, m->B);
    if (tokens)
        for (int b = 0; b < batch; b++)
            if (tokens[b] < 0 || tokens[b] >= m->c.vocab) return fail(m, QW_ERR_ARG, "token %d outside vocab", tokens[b]);
    qw_status s = check_positions(m, slots, positions, batch);
    if (s) return s;
    int *pin = m->h_pin_i;
    const int MB = m->B;
    if (tokens) memcpy(pin, tokens, sizeof(int) * batch);
    memcpy(pin + MB, positions, sizeof(int) * batch);
    if (slots) memcpy(pin + 2 * MB, slots, sizeof(int) * batch);
    else for (int b = 0; b < batch; b++) pin[2 * MB + b] = b;
    // device layout mirrors the pinned block: d_tokens | d_pos | d_slots (contiguous, see create)
    CK(cudaMemcpyAsync(m->d_tokens, pin, sizeof(int) * 3 * MB, cudaMemcpyHostToDevice, m->st));
    float *dlog = nullptr;
    if (logits_out) dlog = m->logits_all ? m->logits_all + (size_t)m->tp * MB * m->Vl : m->logits;
    if (x_in) CK(cudaMemcpyAsync(m->pf.x_host_stage, x_in, sizeof(float) * batch * m->D, cudaMemcpyHostToDevice, m->st));
    s = device_step(m, tokens ? m->d_tokens : nullptr, x_in ? m->pf.x_host_stage : nullptr, m->d_tokens + 2 * MB,
                    m->d_pos, batch, dlog, m->d_argmax, 0, nullptr, 0);
    if (s) return s;
    CK(cudaMemcpyAsync(pin + 3 * MB, m->d_argmax, sizeof(int) * batch, cudaMemcpyDeviceToHost, m->st));
    if (logits_out) CK(cudaMemcpyAsync(logits_out, dlog, sizeof(float) * batch * m->c.vocab, cudaMemcpyDeviceToHost, m->st));
    CK(cudaStreamSynchronize(m->st));
    if (argmax_out) memcpy(argmax_out, pin + 3 * MB, sizeof(int) * batch);
    return QW_OK;
}

// Prefill on the tensor cores: chunks of up to T rows (batch x chunk positions), flash attention
// over the paged cache, then the last position's rmsnorm + lm_head + argmax per sequence.
qw_status tc_prefill(qw_model *m, const int32_t *tokens, const int32_t *slots, int batch, int seq_len,
                     float *logits_out, int32_t *argmax_out) {
    PrefillBuffers &pf = m->pf;
    std::vector<int> sl(batch);
    for (int b = 0; b < batch; b++) {
        sl[b] = slots ? slots[b] : b;
        if (sl[b] < 0 || sl[b] >= m->B) return fail(m, QW_ERR_ARG, "slot %d out of range", sl[b]);
        for (int b2 = 0; b2 < b; b2++)
            if (sl[b2] == sl[b]) return fail(m, QW_ERR_ARG, "slot %d used twice in one batch", sl[b]);
        for (int p = 0; p < seq_len; p++) {
            int t = tokens[(size_t)b * seq_len + p];
            if (t < 0 || t >= m->c.vocab) return fail(m, QW_ERR_ARG, "token %d outside vocab", t);
        }
        TRY(reserve_pages(m, sl[b], seq_len));
    }
    const int Lc = std::max(1, std::min(seq_len, m->T / batch));
    const int Tmax = m->T;
    int *pin = pf.h_pin;
    const float *pending = nullptr;
    bool seq_par = false;
    int L = 0;
    m->launches = 0;
    for (int p0 = 0; p0 < seq_len; p0 += Lc) {
        L = std::min(Lc, seq_len - p0);
        const int T = batch * L;
        CK(cudaStreamSynchronize(m->st));  // the pinned staging of the previous chunk has been consumed
        for (int b = 0; b < batch; b++) {
            pin[3 * Tmax + b] = sl[b];
            for (int i = 0; i < L; i++) {
                const int r = b * L + i;
                pin[r] = sl[b];
                pin[Tmax + r] = p0 + i;
                pin[2 * Tmax + r] = tokens[(size_t)b * seq_len + p0 + i];
            }
        }
        CK(cudaMemcpyAsync(pf.row_slot, pin, sizeof(int) * (size_t)(3 * Tmax + batch), cudaMemcpyHostToDevice, m->st));
        TRY(tc_layers(m, T, pf.row_tok, nullptr, pf.row_slot, pf.row_pos, true, batch, p0, L, pf.seq_slots, &pending,
                      nullptr, &seq_par));
    }
    // last position of every sequence: row b*L + L-1 of the final chunk
    float *dlog = nullptr;
    if (logits_out) dlog = m->logits_all ? m->logits_all + (size_t)m->tp * m->B * m->Vl : m->logits;
    const float *xl = m->xa, *pl = pending;
    size_t ld = (size_t)L * m->D;
    if (seq_par) {
        // the residual rows are current only in their owner's row block: each owner puts x + its partial of those
        // rows into a (batch, D) buffer, zeros elsewhere, and a sum over the ranks gives every rank all of them
        const int T = batch * L, Tl = T / m->tp, rb = m->rank * Tl;
        float *rows = pf.x_host_stage;
        LK(zero_launch(rows, (size_t)batch * m->D, m->st));
        for (int b = 0; b < batch; b++) {
            const int r = b * L + L - 1;
            if (r >= rb && r < rb + Tl)
                LK(add_launch(rows + (size_t)b * m->D, m->xa + (size_t)r * m->D, pending + (size_t)(r - rb) * m->D,
                              m->D, m->st));
        }
        TRY(allreduce(m, rows, (size_t)batch * m->D));
        pl = nullptr;
        ld = m->D;
        xl = rows;
    }
    for (int b0 = 0; b0 < batch; b0 += kGemvMaxB) {
        const int nb = std::min(kGemvMaxB, batch - b0);
        const size_t off = seq_par ? (size_t)b0 * m->D : ((size_t)b0 * L + L - 1) * m->D;
        TRY(lm_head_gemv(m, xl + off, (int)ld, pl ? pl + off : nullptr, (int)ld, nb,
                         dlog ? dlog + (size_t)b0 * m->c.vocab : nullptr, m->d_argmax + b0, nullptr, nullptr, 0,
                         nullptr, 0));
    }
    int *hp = m->h_pin_i + 3 * m->B;
    CK(cudaMemcpyAsync(hp, m->d_argmax, sizeof(int) * batch, cudaMemcpyDeviceToHost, m->st));
    if (logits_out)
        CK(cudaMemcpyAsync(logits_out, dlog, sizeof(float) * (size_t)batch * m->c.vocab, cudaMemcpyDeviceToHost, m->st));
    int derr = 0;
    CK(cudaMemcpyAsync(&pin[0], pf.d_err, sizeof(int), cudaMemcpyDeviceToHost, m->st));
    CK(cudaStreamSynchronize(m->st));
    derr = pin[0];
    if (derr) return fail(m, QW_ERR_TIMEOUT, "tensor-core kernel gave up waiting (device error %d)", derr);
    if (argmax_out) memcpy(argmax_out, hp, sizeof(int) * batch);
    return QW_OK;
}

// (B, V) device logits of a step: the rank's own buffer at tp 1, the gathered block otherwise
float *full_logits(qw_model *m) { return m->logits_all ? m->logits_all + (size_t)m->tp * m->B * m->Vl : m->logits; }

// draw the next token of rows 0..batch-1 from (batch, V) logits with the model's sampling settings
qw_status sample_launch(qw_model *m, const float *logits, int batch, int *out, int advance, int *next_tokens,
                        int *positions, int *hist, int hist_ld) {
    SampleArgs a{};
    a.logits = logits; a.ld = m->c.vocab; a.V = m->c.vocab;
    a.temperature = m->samp_temperature; a.top_p = m->samp_top_p; a.mode = m->samp_mode;
    a.r = nullptr; a.rng = m->d_rng; a.scratch = m->d_samp; a.out = out;
    a.advance = advance; a.next_tokens = next_tokens; a.positions = positions; a.hist = hist; a.hist_ld = hist_ld;
    LK(sample_rows_launch(a, batch, m->st));
    return QW_OK;
}

}  // namespace

namespace qw {
// records an error message for qw_last_error from host code outside this file
void model_set_error(qw_model *m, const std::string &msg) {
    if (m) m->err = msg;
}
}  // namespace qw


// ==========================================================================================
// C ABI
// ==========================================================================================
extern "C" {

int32_t qw_abi_version(void) { return QW_ABI_VERSION; }

const char *qw_build_info(void) {
    return "libqwen3_b200 sm_100a; nvcc " QW_STR(__CUDACC_VER_MAJOR__) "." QW_STR(__CUDACC_VER_MINOR__);
}

qw_status qw_get_unique_id(void *out128) {
    if (!out128) return QW_ERR_ARG;
    ncclUniqueId id;
    if (ncclGetUniqueId(&id) != ncclSuccess) return QW_ERR_NCCL;
    memcpy(out128, &id, sizeof id);
    return QW_OK;
}

// A device buffer of `bytes` on every rank that every peer opens through CUDA IPC (peer access over NVLink): the
// handles travel through an NCCL all-gather.  *local is this rank's buffer, peer_maps the opened peer mappings (to
// close), *d_ptrs a device array [tp] of every rank's pointer.
static qw_status open_peer_buffer(qw_model *m, size_t bytes, void **local, std::vector<void *> &peer_maps,
                                  void ***d_ptrs) {
    const int tp = m->tp;
    CK(cudaMalloc(local, bytes));
    CK(cudaMemset(*local, 0, bytes));
    cudaIpcMemHandle_t h;
    CK(cudaIpcGetMemHandle(&h, *local));
    char *d_h = nullptr;
    CK(cudaMalloc((void **)&d_h, sizeof(h) * (tp + 1)));
    CK(cudaMemcpy(d_h + sizeof(h) * tp, &h, sizeof(h), cudaMemcpyHostToDevice));
    ncclResult_t nr = ncclAllGather(d_h + sizeof(h) * tp, d_h, sizeof(h), ncclChar, m->comm, m->st);
    std::vector<cudaIpcMemHandle_t> all(tp);
    cudaError_t e = cudaStreamSynchronize(m->st);
    if (e == cudaSuccess) e = cudaMemcpy(all.data(), d_h, sizeof(h) * tp, cudaMemcpyDeviceToHost);
    cudaFree(d_h);
    if (nr != ncclSuccess) return fail(m, QW_ERR_NCCL, "exchange handles: %s", ncclGetErrorString(nr));
    if (e != cudaSuccess) return fail(m, QW_ERR_CUDA, "exchange handles: %s", cudaGetErrorString(e));
    std::vector<void *> ptrs(tp);
    for (int p = 0; p < tp; p++) {
        if (p == m->rank) { ptrs[p] = *local; continue; }
        void *q = nullptr;
        CK(cudaIpcOpenMemHandle(&q, all[p], cudaIpcMemLazyEnablePeerAccess));
        peer_maps.push_back(q);
        ptrs[p] = q;
    }
    CK(cudaMalloc((void **)d_ptrs, sizeof(void *) * tp));
    CK(cudaMemcpy(*d_ptrs, ptrs.data(), sizeof(void *) * tp, cudaMemcpyHostToDevice));
    return QW_OK;
}

// Exchange buffers of the tensor-parallel step kernel: flags, sums, argmax, two [tp][D] inboxes of 8-byte words.
static qw_status setup_exchange(qw_model *m) {
    const size_t words = 128 + (size_t)4 * m->tp * m->D;
    return open_peer_buffer(m, words * sizeof(unsigned), (void **)&m->xch, m->xch_peer, (void ***)&m->d_xch);
}

// Inboxes of the batched decode step's all-reduce (qw_allreduce.cu): up to max_batch x dim elements.
static qw_status setup_allreduce(qw_model *m) {
    m->ar_cap = (long long)m->B * m->D;
    m->ar_xoff = (allreduce_ll_words(m->ar_cap, m->tp) + 1) & ~1ll;  // 16-byte aligned pairs of words
    const size_t words = (size_t)m->ar_xoff + (size_t)2 * m->B * m->tp;
    const char *fe = getenv("QW_AR_FUSE");
    m->ar_fuse = !(fe && fe[0] == '0');
    const char *pe = getenv("QW_PREFILL_SP");
    m->prefill_sp = !(pe && pe[0] == '0');
    qw_status s = open_peer_buffer(m, words * 8, (void **)&m->ar_buf, m->xch_peer, (void ***)&m->d_ar);
    if (s) return s;
    AL(m->ar_ctr, 2);
    CK(cudaMemset(m->ar_ctr, 0, 2 * sizeof(unsigned)));
    return QW_OK;
}

static qw_status create_impl(qw_model *m, const qw_config *cfg, int device, int tp_rank, int tp_size,
                             const void *nccl_id) {
    const qw_config &c = *cfg;
    if (c.dim <= 0 || c.layers <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.vocab <= 0 || c.seq_len <= 0 ||
        c.hidden_dim <= 0 || c.max_batch <= 0)
        return fail(m, QW_ERR_SHAPE, "non-positive dimension in config");
    if (c.head_dim != 64 && c.head_dim != 128) return fail(m, QW_ERR_UNSUPPORTED, "head_dim %d (64 or 128)", c.head_dim);
    if (c.heads % c.kv_heads) return fail(m, QW_ERR_SHAPE, "heads %d not a multiple of kv_heads %d", c.heads, c.kv_heads);
    int G = c.heads / c.kv_heads;
    if (G < 1 || G > 8 || G == 3 || G == 5)
        return fail(m, QW_ERR_UNSUPPORTED, "heads per kv group %d (1, 2, 4, 6, 7 or 8)", G);
    if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size) return fail(m, QW_ERR_ARG, "tp rank/size %d/%d", tp_rank, tp_size);
    if (c.kv_heads % tp_size || c.vocab % tp_size || c.hidden_dim % (kGuBlock * tp_size))
        return fail(m, QW_ERR_SHAPE, "kv_heads, vocab and hidden_dim/16 must divide by tp=%d", tp_size);
    if (c.dim % 8 || (c.hidden_dim / tp_size) % 8) return fail(m, QW_ERR_SHAPE, "dim and hidden_dim/tp must be multiples of 8");
    if (c.weight_dtype != QW_DTYPE_F32 && c.weight_dtype != QW_DTYPE_BF16) return fail(m, QW_ERR_UNSUPPORTED, "weight dtype");
    if (c.kv_dtype != QW_DTYPE_F32 && c.kv_dtype != QW_DTYPE_BF16) return fail(m, QW_ERR_UNSUPPORTED, "kv dtype");
    if (c.qk_norm < 0 || c.qk_norm > 2) return fail(m, QW_ERR_ARG, "qk_norm mode %d", c.qk_norm);
    if (c.eps <= 0 || c.rope_theta <= 0) return fail(m, QW_ERR_ARG, "eps / rope_theta must be positive");
    m->c = c;
    m->page_size = c.page_size ? c.page_size : 64;
    if (m->page_size < 16 || m->page_size > 256 || (m->page_size & (m->page_size - 1)))
        return fail(m, QW_ERR_ARG, "page_size %d (power of two in [16,256])", m->page_size);
    m->log2_page = 0;
    while ((1 << m->log2_page) < m->page_size) m->log2_page++;
    m->dev = device; m->rank = tp_rank; m->tp = tp_size;
    cudaGetLastError();  // an earlier, unrelated failure of this thread must not be reported as ours

    m->bf16w = c.weight_dtype == QW_DTYPE_BF16; m->wsz = m->bf16w ? 2 : 4;
    m->bf16kv = c.kv_dtype == QW_DTYPE_BF16; m->kvsz = m->bf16kv ? 2 : 4;
    m->D = c.dim; m->Hl = c.heads / tp_size; m->Hkvl = c.kv_heads / tp_size;
    m->Ql = m->Hl * c.head_dim; m->KVl = m->Hkvl * c.head_dim; m->QKVl = m->Ql + 2 * m->KVl;
    m->Fl = c.hidden_dim / tp_size; m->Vl = c.vocab / tp_size; m->v0 = tp_rank * m->Vl;
    m->B = c.max_batch; m->T = std::max(c.max_tokens, c.max_batch);

    CK(cudaSetDevice(device));
    CK(cudaDeviceGetAttribute(&m->num_sms, cudaDevAttrMultiProcessorCount, device));
    CK(cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking));
    if (tp_size > 1) {
        if (!nccl_id) return fail(m, QW_ERR_ARG, "tp_size > 1 needs an NCCL unique id");
        ncclUniqueId id;
        memcpy(&id, nccl_id, sizeof id);
        NK(ncclCommInitRank(&m->comm, tp_size, id, tp_rank));
    }
    const int D = m->D;
    // ---- weights ----
    m->L.resize(c.layers);
    for (int l = 0; l < c.layers; l++) {
        Layer &Ly = m->L[l];
        ALB(Ly.w_qkv, (size_t)m->QKVl * D * m->wsz);
        if (c.has_qkv_bias) AL(Ly.b_qkv, m->QKVl);
        if (c.qk_norm) { AL(Ly.qn, m->Ql); AL(Ly.kn, m->KVl); }
        ALB(Ly.w_o, (size_t)D * m->Ql * m->wsz);
        ALB(Ly.w_gu, (size_t)2 * m->Fl * D * m->wsz);
        ALB(Ly.w_down, (size_t)D * m->Fl * m->wsz);
        AL(Ly.rms_att, D);
        AL(Ly.rms_ffn, D);
    }
    ALB(m->embed, (size_t)c.vocab * D * m->wsz);
    if (c.shared_weights && tp_size == 1) { m->lm = m->embed; m->lm_alias = true; }
    else ALB(m->lm, (size_t)m->Vl * D * m->wsz);
    AL(m->norm_final, D);
    AL(m->freq, (size_t)c.seq_len * (c.head_dim / 2));
    CK(freq_launch(m->freq, c.seq_len, c.head_dim, c.rope_theta, m->st));
    // ---- paged KV ----
    m->max_pages = (c.seq_len + m->page_size - 1) / m->page_size;
    m->num_pages = c.num_pages > 0 ? c.num_pages : m->B * m->max_pages;
    m->layer_kv_elems = (size_t)m->num_pages * m->Hkvl * m->page_size * c.head_dim;
    ALB(m->kpool, m->layer_kv_elems * c.layers * m->kvsz);
    ALB(m->vpool, m->layer_kv_elems * c.layers * m->kvsz);
    CK(cudaMemsetAsync(m->kpool, 0, m->layer_kv_elems * c.layers * m->kvsz, m->st));
    CK(cudaMemsetAsync(m->vpool, 0, m->layer_kv_elems * c.layers * m->kvsz, m->st));
    AL(m->d_page_table, (size_t)m->B * m->max_pages);
    m->h_page_table.assign((size_t)m->B * m->max_pages, 0);
    CK(cudaMemsetAsync(m->d_page_table, 0, sizeof(int) * m->B * m->max_pages, m->st));
    m->slot_pages.assign(m->B, {});
    for (int p = m->num_pages - 1; p >= 0; p--) m->free_pages.push_back(p);
    // ---- activations ----
    const int T = m->T, B = m->B;
    AL(m->xa, (size_t)T * D);
    AL(m->xb, (size_t)T * D);
    if (tp_size > 1) AL(m->part, (size_t)T * D);
    AL(m->qkv, (size_t)T * m->QKVl);
    AL(m->attn, (size_t)T * m->Ql);
    AL(m->hbuf, (size_t)T * m->Fl);
    AL(m->part_o, (size_t)B * m->Hl * m->maxsplit * c.head_dim);
    AL(m->part_ml, (size_t)B * m->Hl * m->maxsplit * 2);
    AL(m->qk_ss, (size_t)B * 2);
    AL(m->counters, (size_t)B * m->Hkvl);
    CK(cudaMemsetAsync(m->counters, 0, sizeof(unsigned) * B * m->Hkvl, m->st));
    AL(m->am_counter, 1);
    CK(cudaMemsetAsync(m->am_counter, 0, sizeof(unsigned), m->st));
    AL(m->am_pval, (size_t)m->num_sms * 16 * kGemvMaxB);
    AL(m->am_pidx, (size_t)m->num_sms * 16 * kGemvMaxB);
    AL(m->am_val, B);
    AL(m->am_idx, B);
    AL(m->am_val_all, (size_t)B * tp_size);
    AL(m->am_idx_all, (size_t)B * tp_size);
    AL(m->logits, (size_t)B * m->Vl);
    // logits_all: gathered shards [tp][B][Vl] followed by a (B, V) assembled block
    if (tp_size > 1) AL(m->logits_all, (size_t)2 * tp_size * B * m->Vl);
    AL(m->d_tokens, (size_t)3 * B);  // tokens | positions | slots
    m->d_pos = m->d_tokens + B;
    m->d_slots = m->d_tokens + 2 * B;
    {
        std::vector<int> ident(B);
        for (int b = 0; b < B; b++) ident[b] = b;
        CK(cudaMemcpy(m->d_slots, ident.data(), sizeof(int) * B, cudaMemcpyHostToDevice));
    }
    AL(m->d_argmax, B);
    CK(cudaHostAlloc((void **)&m->h_pin_i, sizeof(int) * 4 * B, cudaHostAllocDefault));
    qw_status s = prefill_alloc(m->pf, c, m->T, m->B, m->Ql, m->KVl, m->Fl, m->D);
    if (s) return fail(m, s, "prefill buffers: %s", cudaGetErrorString(cudaGetLastError()));
    if (m->pf.tc) {
        CK(tc_prepare());
        CK(prefill_kernels_prepare());
        if (c.head_dim == 128) {
            // causal prefill attention on tcgen05 (QW_TC_ATTN=0: the mma.sync kernel, for comparison)
            const char *ev = getenv("QW_TC_ATTN");
            m->tc_attn = !ev || atoi(ev) != 0;
            if (m->tc_attn) CK(flash_prefill_tc_prepare());
        }
        AL(m->gu_split, (size_t)B * 2 * m->Fl);
        AL(m->qkv_split, (size_t)B * m->QKVl);
        AL(m->part_split, (size_t)B * m->D);
        CK(cudaMemset(m->part_split, 0, sizeof(float) * (size_t)B * m->D));
        CK(cudaMemset(m->gu_split, 0, sizeof(float) * (size_t)B * 2 * m->Fl));
        CK(cudaMemset(m->qkv_split, 0, sizeof(float) * (size_t)B * m->QKVl));
        AL(m->cand_val, (size_t)B * ((m->Vl + 127) / 128 * 4));
        AL(m->cand_idx, (size_t)B * ((m->Vl + 127) / 128 * 4));
        if (tp_size > 1) {
            // batched decode all-reduces over NVLink (QW_AR_NCCL=1: NCCL, for comparison)
            const char *ev = getenv("QW_AR_NCCL");
            if (!ev || atoi(ev) == 0) {
                qw_status st = setup_allreduce(m);
                if (st) return st;
            }
        }
    }
    // the persistent step kernel for batch-1 decode with bf16 weights at any tp (decode_kernels 0 or 2) when the
    // geometry fits it; under tensor parallelism its all-reduces are flag-in-data exchanges over NVLink
    if (m->bf16w && c.decode_kernels != 1) {
        StepArgs &sa = m->step;
        sa.layers = c.layers; sa.D = D; sa.F = m->Fl; sa.V = m->Vl; sa.H = m->Hl; sa.Hkv = m->Hkvl; sa.d = c.head_dim;
        sa.kv_bf16 = m->bf16kv;
        size_t smem = 0;
        int coop = 0;
        CK(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device));
        if (coop && step_layout(sa, m->num_sms, &smem)) {
            CK(step_prepare(m->bf16kv, c.head_dim, m->Hl / m->Hkvl, tp_size > 1, smem));
            int occ = 0;
            CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                &occ, step_kernel_fn(m->bf16kv, c.head_dim, m->Hl / m->Hkvl, tp_size > 1), kStepBlockThreads, smem));
            if (occ >= 1) {
                m->use_step = true;
                sa.norm_final = m->norm_final; sa.eps = (float)c.eps; sa.scale = (float)(1.0 / sqrt((double)c.head_dim));
                sa.qk_mode = c.qk_norm; sa.freq = m->freq; sa.page_table = m->d_page_table; sa.max_pages = m->max_pages;
                sa.page_size = m->page_size; sa.log2_page = m->log2_page;
                sa.x = m->xa; sa.qkv = m->qkv; sa.attn = m->attn;
                AL(m->gu, (size_t)2 * m->Fl);
                sa.gu = m->gu;
                sa.part_o = m->part_o; sa.part_ml = m->part_ml;
                sa.am_val = m->am_pval; sa.am_idx = m->am_pidx;
                // per-step state, zeroed by one memset before every launch: barrier counter,
                // (layers, 2) q/k sums of squares, (layers, Hkv) attention split arrivals
                m->step_zero_words = 1 + 2 * (size_t)c.layers + (size_t)c.layers * m->Hkvl;
                ALB(m->d_bar, sizeof(unsigned) * m->step_zero_words);
                sa.bar = m->d_bar;
                sa.ss = reinterpret_cast<float *>(m->d_bar + 1);
                sa.counters = m->d_bar + 1 + 2 * c.layers;
                AL(m->d_trace, (size_t)2 * (5 * c.layers + 2) + (size_t)8 * c.layers);
                sa.err = m->pf.d_err;
                {
                    const char *ev = getenv("QW_STEP_EVICT");
                    sa.evict_first = ev ? atoi(ev) : 1;
                    const char *rc = getenv("QW_STEP_ROWCOPY");
                    sa.row_copies = rc ? atoi(rc) : 0;
                }
                {
                    int khz = 0;
                    CK(cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, device));
                    const long long us = c.wait_limit_us > 0 ? c.wait_limit_us : 2000000;
                    sa.wait_cycles = (unsigned long long)us * (unsigned long long)(khz > 0 ? khz : 2000000) / 1000ull;
                    sa.stall_cta = c.test_stall_cta > 0 ? c.test_stall_cta - 1 : -1;
                }
                sa.tp = tp_size; sa.rank = tp_rank; sa.v0 = m->v0;
                sa.q_total = c.heads * c.head_dim; sa.kv_total = c.kv_heads * c.head_dim;
                AL(m->d_persist, 2);
                CK(cudaMemset(m->d_persist, 0, 2 * sizeof(unsigned)));
                sa.gen = m->d_persist;
                if (tp_size > 1) {
                    qw_status st = setup_exchange(m);
                    if (st) return st;
                    sa.xch = m->d_xch;
                }
            }
        }
    }
    CK(cudaStreamSynchronize(m->st));
    return QW_OK;
}

qw_status qw_create(const qw_config *cfg, int32_t device, int32_t tp_rank, int32_t tp_size, const void *nccl_unique_id,
                    qw_model **out) {
    if (!cfg || !out) return QW_ERR_ARG;
    *out = nullptr;
    qw_model *m = new qw_model();
    qw_status s = create_impl(m, cfg, device, tp_rank, tp_size, nccl_unique_id);
    if (s) {
        // keep the message visible through a thread-local fallback
        static thread_local std::string last;
        last = m->err;
        fprintf(stderr, "qw_create: %s\n", m->err.c_str());
        qw_destroy(m);
        return s;
    }
    *out = m;
    return QW_OK;
}

qw_status qw_load_tensor(qw_model *m, const char *key, qw_dtype dtype, const int64_t *dims, int32_t ndims,
                         const void *host_ptr) {
    if (!m || !key || !host_ptr || (ndims > 0 && !dims)) return m ? fail(m, QW_ERR_ARG, "null argument") : QW_ERR_ARG;
    if (dtype != QW_DTYPE_F32 && dtype != QW_DTYPE_BF16 && dtype != QW_DTYPE_F64) return fail(m, QW_ERR_ARG, "dtype %d", dtype);
    CK(cudaSetDevice(m->dev));
    Target t;
    int r = resolve(m, key, t);
    if (r == -1) return fail(m, QW_ERR_KEY, "unknown state-dict key '%s'", key);
    if (r == -2) return QW_OK;  // tensor not used by this configuration (e.g. tied lm_head)
    long long numel = 1;
    for (int i = 0; i < ndims; i++) numel *= dims[i];
    long long want = t.full_rows * t.full_cols;
    bool shape_ok = numel == want;
    if (shape_ok && ndims == 2 && t.full_rows > 1 && t.full_cols > 1) shape_ok = dims[0] == t.full_rows && dims[1] == t.full_cols;
    if (!shape_ok) return fail(m, QW_ERR_SHAPE, "'%s': %lld elements, expected %lld x %lld", key, numel, t.full_rows, t.full_cols);
    size_t es = dtype == QW_DTYPE_F32 ? 4 : dtype == QW_DTYPE_BF16 ? 2 : 8;
    void *stage = nullptr;
    size_t bytes = (size_t)t.rows * t.cols * es;
    CK(cudaMalloc(&stage, bytes));
    const char *src = (const char *)host_ptr + ((size_t)t.r0 * t.full_cols + t.c0) * es;
    cudaError_t e = cudaMemcpy2DAsync(stage, t.cols * es, src, (size_t)t.full_cols * es, t.cols * es, t.rows,
                                      cudaMemcpyHostToDevice, m->st);
    qw_status s = QW_OK;
    if (e != cudaSuccess) s = fail(m, QW_ERR_CUDA, "copy '%s': %s", key, cudaGetErrorString(e));
    if (!s) s = place(m, t, stage, dtype == QW_DTYPE_F32 ? 0 : dtype == QW_DTYPE_BF16 ? 1 : 2, t.cols, false, 0, 0.f);
    e = cudaStreamSynchronize(m->st);
    cudaFree(stage);
    if (s) return s;
    if (e != cudaSuccess) return fail(m, QW_ERR_CUDA, "place '%s': %s", key, cudaGetErrorString(e));
    *t.loaded |= t.bit;
    m->finalized = false;
    return QW_OK;
}

qw_status qw_init_synthetic(qw_model *m, uint64_t seed, float stdv) {
    if (!m) return QW_ERR_ARG;
    CK(cudaSetDevice(m->dev));
    const qw_config &c = m->c;
    std::vector<std::string> keys = {"model.embed_tokens.weight", "model.norm.weight"};
    if (!c.shared_weights) keys.push_back("lm_head.weight");
    for (int l = 0; l < c.layers; l++)
        for (int k = 0; k < K_NUM_LAYER_KINDS; k++) keys.push_back("model.layers." + std::to_string(l) + "." + kLayerNames[k]);
    for (auto &k : keys) {
        Target t;
        int r = resolve(m, k.c_str(), t);
        if (r) continue;
        qw_status s = place(m, t, nullptr, 0, 0, true, seed, stdv);
        if (s) return s;
        *t.loaded |= t.bit;
    }
    CK(cudaStreamSynchronize(m->st));
    m->finalized = false;
    return QW_OK;
}

qw_status qw_finalize_weights(qw_model *m) {
    if (!m) return QW_ERR_ARG;
    CK(cudaSetDevice(m->dev));
    const qw_config &c = m->c;
    uint32_t need_top = (1u << K_EMBED) | (1u << K_NORM) | (c.shared_weights ? 0u : (1u << K_LMHEAD));
    if ((m->top_loaded & need_top) != need_top) return fail(m, QW_ERR_STATE, "missing embed_tokens / norm / lm_head weights");
    uint32_t need = required_layer_bits(c);
    for (int l = 0; l < c.layers; l++)
        if ((m->L[l].loaded & need) != need) {
            for (int k = 0; k < K_NUM_LAYER_KINDS; k++)
                if ((need >> k & 1) && !(m->L[l].loaded >> k & 1))
                    return fail(m, QW_ERR_STATE, "missing model.layers.%d.%s", l, kLayerNames[k]);
        }
    if (c.shared_weights && !m->lm_alias)
        CK(cudaMemcpyAsync(m->lm, (char *)m->embed + (size_t)m->v0 * m->D * m->wsz, (size_t)m->Vl * m->D * m->wsz,
                           cudaMemcpyDeviceToDevice, m->st));
    if (m->use_step && !m->d_step_layers) {
        std::vector<StepLayer> sl(c.layers);
        for (int l = 0; l < c.layers; l++) {
            const Layer &Ly = m->L[l];
            sl[l].w_qkv = (const __nv_bfloat16 *)Ly.w_qkv; sl[l].w_o = (const __nv_bfloat16 *)Ly.w_o;
            sl[l].w_gu = (const __nv_bfloat16 *)Ly.w_gu; sl[l].w_down = (const __nv_bfloat16 *)Ly.w_down;
            sl[l].b_qkv = Ly.b_qkv; sl[l].qn = Ly.qn; sl[l].kn = Ly.kn; sl[l].rms_att = Ly.rms_att;
            sl[l].rms_ffn = Ly.rms_ffn;
            sl[l].kc = (char *)m->kpool + (size_t)l * m->layer_kv_elems * m->kvsz;
            sl[l].vc = (char *)m->vpool + (size_t)l * m->layer_kv_elems * m->kvsz;
        }
        AL(m->d_step_layers, c.layers);
        CK(cudaMemcpy(m->d_step_layers, sl.data(), sizeof(StepLayer) * c.layers, cudaMemcpyHostToDevice));
        m->step.L = m->d_step_layers;
        m->step.lm = (const __nv_bfloat16 *)m->lm;
        m->step.embed = (const __nv_bfloat16 *)m->embed;
    }
    CK(cudaStreamSynchronize(m->st));
    m->finalized = true;
    return QW_OK;
}

qw_status qw_reset(qw_model *m, int32_t slot) {
    if (!m) return QW_ERR_ARG;
    if (slot < -1 || slot >= m->B) return fail(m, QW_ERR_ARG, "slot %d", slot);
    for (int s = 0; s < m->B; s++)
        if (slot == -1 || s == slot) release_slot(m, s);
    return QW_OK;
}

qw_status qw_reserve(qw_model *m, int32_t slot, int32_t n_positions) {
    if (!m) return QW_ERR_ARG;
    CK(cudaSetDevice(m->dev));
    return reserve_pages(m, slot, n_positions);
}

qw_status qw_decode_step(qw_model *m, const int32_t *tokens, const int32_t *slots, const int32_t *positions,
                         int32_t batch, float *logits_out, int32_t *argmax_out) {
    if (!m) return QW_ERR_ARG;
    if (!tokens) return fail(m, QW_ERR_ARG, "null tokens");
    CK(cudaSetDevice(m->dev));
    return host_step(m, tokens, nullptr, slots, positions, batch, logits_out, argmax_out);
}

qw_status qw_forward_hidden(qw_model *m, const float *x_in, const int32_t *slots, const int32_t *positions,
                            int32_t batch, float *logits_out, int32_t *argmax_out) {
    if (!m) return QW_ERR_ARG;
    if (!x_in) return fail(m, QW_ERR_ARG, "null x_in");
    CK(cudaSetDevice(m->dev));
    return host_step(m, nullptr, x_in, slots, positions, batch, logits_out, argmax_out);
}

qw_status qw_decode_step_device(qw_model *m, int32_t *d_tokens, const int32_t *d_slots, int32_t *d_positions,
                                int32_t batch, float *d_logits, int32_t *d_argmax, int32_t advance) {
    if (!m) return QW_ERR_ARG;
    if (!d_tokens || !d_positions) return fail(m, QW_ERR_ARG, "null device pointer");
    CK(cudaSetDevice(m->dev));
    return device_step(m, d_tokens, nullptr, d_slots, d_positions, batch, d_logits, d_argmax, advance, nullptr, 0);
}

qw_status qw_capture_decode(qw_model *m, int32_t *d_tokens, const int32_t *d_slots, int32_t *d_positions, int32_t batch,
                            float *d_logits, int32_t *d_argmax) {
    if (!m) return QW_ERR_ARG;
    CK(cudaSetDevice(m->dev));
    if (m->graph) { cudaGraphExecDestroy(m->graph); m->graph = nullptr; }
    cudaGraph_t g;
    CK(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal));
    qw_status s = device_step(m, d_tokens, nullptr, d_slots, d_positions, batch, d_logits, d_argmax, 1, nullptr, 0);
    cudaError_t e = cudaStreamEndCapture(m->st, &g);
    if (s) return s;
    if (e != cudaSuccess) return fail(m, QW_ERR_CUDA, "capture: %s", cudaGetErrorString(e));
    e = cudaGraphInstantiate(&m->graph, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return fail(m, QW_ERR_CUDA, "instantiate: %s", cudaGetErrorString(e));
    return QW_OK;
}

qw_status qw_replay_decode(qw_model *m, int32_t times) {
    if (!m) return QW_ERR_ARG;
    if (!m->graph) return fail(m, QW_ERR_STATE, "no captured decode graph");
    CK(cudaSetDevice(m->dev));
    for (int i = 0; i < times; i++) CK(cudaGraphLaunch(m->graph, m->st));
    return QW_OK;
}

qw_status qw_prefill(qw_model *m, const int32_t *tokens, const int32_t *slots, int32_t batch, int32_t seq_len,
                     float *logits_out, int32_t *argmax_out) {
    if (!m) return QW_ERR_ARG;
    if (!tokens) return fail(m, QW_ERR_ARG, "null tokens");
    if (batch < 1 || batch > m->B || seq_len < 1 || seq_len > m->c.seq_len)
        return fail(m, QW_ERR_SHAPE, "prefill batch %d x %d", batch, seq_len);
    CK(cudaSetDevice(m->dev));
    if (!m->finalized) return fail(m, QW_ERR_STATE, "weights not finalized");
    if (m->pf.tc) return tc_prefill(m, tokens, slots, batch, seq_len, logits_out, argmax_out);
    // Token-by-token prefill through the decode kernels (the reference's own schedule; the fp32 path).
    std::vector<int> tok(batch), pos(batch);
    for (int p = 0; p < seq_len; p++) {
        for (int b = 0; b < batch; b++) { tok[b] = tokens[(size_t)b * seq_len + p]; pos[b] = p; }
        bool last = p == seq_len - 1;
        qw_status s = host_step(m, tok.data(), nullptr, slots, pos.data(), batch, last ? logits_out : nullptr,
                                last ? argmax_out : nullptr);
        if (s) return s;
    }
    return QW_OK;
}

// Sampled generation (AutoregressiveModel.next with a temperature): the prompt's last logits give the
// first generated token; every later step writes its logits and the sampling kernel feeds the drawn token
// back and advances the position, all on the device.
static qw_status generate_sampled(qw_model *m, const int32_t *prompts, int32_t batch, int32_t prompt_len,
                                  int32_t steps, int32_t *tokens_out) {
    const int V = m->c.vocab;
    std::vector<float> lg((size_t)batch * V);
    for (int b = 0; b < batch; b++) release_slot(m, b);
    for (int b = 0; b < batch; b++) {
        qw_status s = reserve_pages(m, b, steps);
        if (s) return s;
    }
    qw_status s = qw_prefill(m, prompts, nullptr, batch, prompt_len, lg.data(), nullptr);
    if (s) return s;
    for (int b = 0; b < batch; b++)
        for (int i = 0; i < prompt_len; i++) tokens_out[(size_t)b * steps + i] = prompts[(size_t)b * prompt_len + i];
    if (steps == prompt_len) return QW_OK;
    float *dlog = full_logits(m);
    int *hist = nullptr;
    AL(hist, (size_t)batch * (steps + 1));
    std::vector<int> pos(batch, prompt_len - 1);
    CK(cudaMemcpyAsync(dlog, lg.data(), sizeof(float) * lg.size(), cudaMemcpyHostToDevice, m->st));
    CK(cudaMemcpyAsync(m->d_pos, pos.data(), sizeof(int) * batch, cudaMemcpyHostToDevice, m->st));
    // the first generated token: its position is prompt_len (the draw advances d_pos to it)
    s = sample_launch(m, dlog, batch, nullptr, 1, m->d_tokens, m->d_pos, hist, steps + 1);
    for (int st = prompt_len; !s && st < steps - 1; st++) {
        s = device_step(m, m->d_tokens, nullptr, m->d_slots, m->d_pos, batch, dlog, m->d_argmax, 0, nullptr, 0);
        if (!s) s = sample_launch(m, dlog, batch, nullptr, 1, m->d_tokens, m->d_pos, hist, steps + 1);
    }
    std::vector<int> h((size_t)batch * (steps + 1));
    cudaError_t e = cudaSuccess;
    if (!s) e = cudaMemcpyAsync(h.data(), hist, sizeof(int) * h.size(), cudaMemcpyDeviceToHost, m->st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->st);
    cudaFree(hist);
    if (s) return s;
    if (e != cudaSuccess) return fail(m, QW_ERR_CUDA, "generate: %s", cudaGetErrorString(e));
    for (int b = 0; b < batch; b++)
        for (int i = prompt_len; i < steps; i++) tokens_out[(size_t)b * steps + i] = h[(size_t)b * (steps + 1) + i];
    return QW_OK;
}

qw_status qw_generate(qw_model *m, const int32_t *prompts, int32_t batch, int32_t prompt_len, int32_t steps,
                      int32_t *tokens_out) {
    if (!m) return QW_ERR_ARG;
    if (!prompts || !tokens_out) return fail(m, QW_ERR_ARG, "null prompts / tokens_out");
    if (prompt_len < 1 || steps < prompt_len || steps > m->c.seq_len)
        return fail(m, QW_ERR_SHAPE, "generate: prompt_len %d steps %d (seq_len %d)", prompt_len, steps, m->c.seq_len);
    if (batch < 1 || batch > m->B) return fail(m, QW_ERR_SHAPE, "batch %d", batch);
    CK(cudaSetDevice(m->dev));
    for (int b = 0; b < batch; b++) {
        release_slot(m, b);
        qw_status s = reserve_pages(m, b, steps);
        if (s) return s;
    }
    std::vector<int> next(batch);
    qw_status s = qw_prefill(m, prompts, nullptr, batch, prompt_len, nullptr, next.data());
    if (s) return s;
    for (int b = 0; b < batch; b++)
        for (int i = 0; i < prompt_len; i++) tokens_out[(size_t)b * steps + i] = prompts[(size_t)b * prompt_len + i];
    if (steps == prompt_len) return QW_OK;
    if (m->samp_temperature > 0.0) return generate_sampled(m, prompts, batch, prompt_len, steps, tokens_out);
    // device-resident greedy loop: the argmax epilogue feeds the next step and advances positions
    int *hist = nullptr;
    AL(hist, (size_t)batch * (steps + 1));
    std::vector<int> pos(batch, prompt_len);
    CK(cudaMemcpyAsync(m->d_tokens, next.data(), sizeof(int) * batch, cudaMemcpyHostToDevice, m->st));
    CK(cudaMemcpyAsync(m->d_pos, pos.data(), sizeof(int) * batch, cudaMemcpyHostToDevice, m->st));
    for (int b = 0; b < batch; b++)
        CK(cudaMemcpyAsync(hist + (size_t)b * (steps + 1) + prompt_len, &next[b], sizeof(int), cudaMemcpyHostToDevice, m->st));
    for (int st = prompt_len; st < steps; st++) {
        s = device_step(m, m->d_tokens, nullptr, m->d_slots, m->d_pos, batch, nullptr, m->d_argmax, 1, hist, steps + 1);
        if (s) { cudaFree(hist); return s; }
    }
    std::vector<int> h((size_t)batch * (steps + 1));
    cudaError_t e = cudaMemcpyAsync(h.data(), hist, sizeof(int) * h.size(), cudaMemcpyDeviceToHost, m->st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->st);
    cudaFree(hist);
    if (e != cudaSuccess) return fail(m, QW_ERR_CUDA, "generate: %s", cudaGetErrorString(e));
    for (int b = 0; b < batch; b++)
        for (int i = prompt_len; i < steps; i++) tokens_out[(size_t)b * steps + i] = h[(size_t)b * (steps + 1) + i];
    return QW_OK;
}

qw_status qw_profile_prefill(qw_model *m, const int32_t *tokens, const int32_t *slots, int32_t batch, int32_t seq_len,
                             float *ms_out, int32_t *kinds_out, int32_t cap, int32_t *n_out) {
    if (!m || !tokens || !ms_out || !kinds_out || !n_out || cap < 1)
        return m ? fail(m, QW_ERR_ARG, "null argument") : QW_ERR_ARG;
    if (!m->pf.tc) return fail(m, QW_ERR_UNSUPPORTED, "prefill profiling needs the tensor-core path (bf16)");
    if (batch < 1 || batch > m->B || seq_len < 1) return fail(m, QW_ERR_SHAPE, "batch %d / seq_len %d", batch, seq_len);
    CK(cudaSetDevice(m->dev));
    while ((int)m->prof_ev.size() < 2 * cap) {
        cudaEvent_t e;
        CK(cudaEventCreate(&e));
        m->prof_ev.push_back(e);
    }
    m->prof_kinds.assign(cap, 0);
    m->prof_n = 0;
    m->prof_on = true;
    qw_status s = tc_prefill(m, tokens, slots, batch, seq_len, nullptr, nullptr);
    m->prof_on = false;
    if (s) return s;
    CK(cudaStreamSynchronize(m->st));
    for (int i = 0; i < m->prof_n; i++) {
        CK(cudaEventElapsedTime(&ms_out[i], m->prof_ev[2 * i], m->prof_ev[2 * i + 1]));
        kinds_out[i] = m->prof_kinds[i];
    }
    *n_out = m->prof_n;
    return QW_OK;
}

qw_status qw_profile_decode(qw_model *m, int32_t batch, float *ms_out, int32_t *kinds_out, int32_t cap,
                            int32_t *n_out) {
    if (!m || !ms_out || !kinds_out || !n_out || cap < 1) return m ? fail(m, QW_ERR_ARG, "null argument") : QW_ERR_ARG;
    if (batch < 1 || batch > m->B) return fail(m, QW_ERR_SHAPE, "batch %d", batch);
    CK(cudaSetDevice(m->dev));
    while ((int)m->prof_ev.size() < 2 * cap) {
        cudaEvent_t e;
        CK(cudaEventCreate(&e));
        m->prof_ev.push_back(e);
    }
    m->prof_kinds.assign(cap, 0);
    m->prof_n = 0;
    // keep the GPU busy while the host enqueues the step, so event pairs bracket device time only
    CK(hold_launch(20ull * 1000 * 1000, m->st));
    m->prof_on = true;
    // positions / tokens / slots are the model's own device buffers (current contents)
    qw_status s = device_step(m, m->d_tokens, nullptr, m->d_slots, m->d_pos, batch, nullptr, m->d_argmax, 0, nullptr, 0);
    m->prof_on = false;
    if (s) return s;
    CK(cudaStreamSynchronize(m->st));
    if (m->use_step && batch == 1 && m->prof_n == 1) {
        // one persistent kernel: report its phases from CTA 0's timestamps -- the work of each
        // phase under its kernel class, the wait in the grid barrier after it as QW_KERNEL_OTHER
        const int nb = 5 * m->c.layers;
        std::vector<unsigned long long> tr((size_t)2 * nb + 2);
        CK(cudaMemcpy(tr.data(), m->d_trace, sizeof(unsigned long long) * tr.size(), cudaMemcpyDeviceToHost));
        const int kinds[5] = {QW_KERNEL_QKV, QW_KERNEL_ATTN, QW_KERNEL_O, QW_KERNEL_GATE_UP, QW_KERNEL_DOWN};
        int n = 0;
        for (int i = 0; i <= nb && n + 2 <= cap; i++) {
            ms_out[n] = (float)((double)(tr[2 * i + 1] - tr[2 * i]) * 1e-6);
            kinds_out[n++] = i < nb ? kinds[i % 5] : QW_KERNEL_LM_HEAD;
            if (i < nb) {
                ms_out[n] = (float)((double)(tr[2 * i + 2] - tr[2 * i + 1]) * 1e-6);
                kinds_out[n++] = QW_KERNEL_OTHER;
            }
        }
        if (getenv("QW_TRACE_ATTN")) {
            // development aid: mean sub-phase times of CTA 0's attention item over the layers
            std::vector<unsigned long long> at((size_t)8 * m->c.layers);
            CK(cudaMemcpy(at.data(), m->d_trace + tr.size(), sizeof(unsigned long long) * at.size(),
                          cudaMemcpyDeviceToHost));
            double sum[7] = {0};
            for (int l = 0; l < m->c.layers; l++) {
                const unsigned long long start = tr[2 * (5 * l) + 2], end = tr[2 * (5 * l + 1) + 1];
                unsigned long long prev = start;
                for (int k = 0; k < 6; k++) {
                    const unsigned long long t = at[(size_t)l * 8 + k];
                    sum[k] += t >= prev ? (double)(t - prev) : 0.0;
                    if (t >= prev) prev = t;
                }
                sum[6] += end >= prev ? (double)(end - prev) : 0.0;
            }
            fprintf(stderr, "attention sub-phases (us, mean of %d layers): qk-sums %.2f  q/k/v %.2f  rope+kv-write %.2f  "
                    "keys %.2f  warp-merge+partials %.2f  split-wait %.2f  merge %.2f\n", m->c.layers,
                    sum[0] / m->c.layers * 1e-3, sum[1] / m->c.layers * 1e-3, sum[2] / m->c.layers * 1e-3,
                    sum[3] / m->c.layers * 1e-3, sum[4] / m->c.layers * 1e-3, sum[5] / m->c.layers * 1e-3,
                    sum[6] / m->c.layers * 1e-3);
        }
        float ms = 0.f;
        CK(cudaEventElapsedTime(&ms, m->prof_ev[0], m->prof_ev[1]));
        if (n < cap) { ms_out[n] = ms; kinds_out[n++] = QW_KERNEL_STEP; }
        *n_out = n;
        return QW_OK;
    }
    for (int i = 0; i < m->prof_n; i++) {
        float ms = 0.f;
        CK(cudaEventElapsedTime(&ms, m->prof_ev[2 * i], m->prof_ev[2 * i + 1]));
        ms_out[i] = ms;
        kinds_out[i] = m->prof_kinds[i];
    }
    *n_out = m->prof_n;
    return QW_OK;
}

qw_status qw_set_device_inputs(qw_model *m, const int32_t *tokens, const int32_t *positions, int32_t batch) {
    if (!m || !tokens || !positions) return m ? fail(m, QW_ERR_ARG, "null argument") : QW_ERR_ARG;
    if (batch < 1 || batch > m->B) return fail(m, QW_ERR_SHAPE, "batch %d", batch);
    CK(cudaSetDevice(m->dev));
    qw_status s = check_positions(m, nullptr, positions, batch);
    if (s) return s;
    CK(cudaMemcpy(m->d_tokens, tokens, sizeof(int) * batch, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(m->d_pos, positions, sizeof(int) * batch, cudaMemcpyHostToDevice));
    return QW_OK;
}

qw_status qw_set_sampling(qw_model *m, double temperature, double top_p, int64_t seed, int32_t mode) {
    if (!m) return QW_ERR_ARG;
    if (mode != 0 && mode != 1) return fail(m, QW_ERR_ARG, "sampling mode %d (0 or 1)", mode);
    if (!(top_p > 0.0)) return fail(m, QW_ERR_ARG, "top_p must be positive");
    CK(cudaSetDevice(m->dev));
    if (!m->d_rng) {
        AL(m->d_rng, m->B);
        AL(m->d_samp, (size_t)m->B * m->c.vocab);
    }
    std::vector<unsigned long long> st(m->B);
    for (int b = 0; b < m->B; b++) st[b] = java_random_state(seed + b);  // new Random(seed + slot)
    CK(cudaMemcpy(m->d_rng, st.data(), sizeof(unsigned long long) * m->B, cudaMemcpyHostToDevice));
    m->samp_temperature = temperature;
    m->samp_top_p = top_p;
    m->samp_mode = mode;
    return QW_OK;
}

qw_status qw_decode_sample(qw_model *m, const int32_t *tokens, const int32_t *slots, const int32_t *positions,
                           int32_t batch, int32_t *tokens_out) {
    if (!m) return QW_ERR_ARG;
    if (!tokens || !positions || !tokens_out) return fail(m, QW_ERR_ARG, "null argument");
    if (!m->finalized) return fail(m, QW_ERR_STATE, "weights not finalized");
    if (batch < 1 || batch > m->B) return fail(m, QW_ERR_SHAPE, "batch %d outside [1,%d]", batch, m->B);
    if (m->samp_temperature > 0.0 && !m->d_rng) return fail(m, QW_ERR_STATE, "sampling state not set");
    CK(cudaSetDevice(m->dev));
    for (int b = 0; b < batch; b++)
        if (tokens[b] < 0 || tokens[b] >= m->c.vocab) return fail(m, QW_ERR_ARG, "token %d outside vocab", tokens[b]);
    qw_status s = check_positions(m, slots, positions, batch);
    if (s) return s;
    int *pin = m->h_pin_i;
    const int MB = m->B;
    memcpy(pin, tokens, sizeof(int) * batch);
    memcpy(pin + MB, positions, sizeof(int) * batch);
    if (slots) memcpy(pin + 2 * MB, slots, sizeof(int) * batch);
    else for (int b = 0; b < batch; b++) pin[2 * MB + b] = b;
    CK(cudaMemcpyAsync(m->d_tokens, pin, sizeof(int) * 3 * MB, cudaMemcpyHostToDevice, m->st));
    float *dlog = full_logits(m);
    if (m->samp_temperature > 0.0) {
        s = device_step(m, m->d_tokens, nullptr, m->d_tokens + 2 * MB, m->d_pos, batch, dlog, m->d_argmax, 0, nullptr, 0);
        if (!s) s = sample_launch(m, dlog, batch, m->d_argmax, 0, nullptr, nullptr, nullptr, 0);
    } else {
        s = device_step(m, m->d_tokens, nullptr, m->d_tokens + 2 * MB, m->d_pos, batch, nullptr, m->d_argmax, 0, nullptr, 0);
    }
    if (s) return s;
    CK(cudaMemcpyAsync(pin + 3 * MB, m->d_argmax, sizeof(int) * batch, cudaMemcpyDeviceToHost, m->st));
    CK(cudaStreamSynchronize(m->st));
    memcpy(tokens_out, pin + 3 * MB, sizeof(int) * batch);
    return QW_OK;
}

qw_status qw_synchronize(qw_model *m) {
    if (!m) return QW_ERR_ARG;
    CK(cudaSetDevice(m->dev));
    CK(cudaStreamSynchronize(m->st));
    // a bounded wait inside a kernel that gave up records its site in the device error word:
    // 1 weight slot, 2 grid barrier, 3 attention split merge, 4 cross-rank barrier, 5 final argmax exchange
    int derr = 0;
    CK(cudaMemcpy(&derr, m->pf.d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (derr) return fail(m, QW_ERR_TIMEOUT, "a device-side wait gave up (site %d)", derr);
    return QW_OK;
}

void *qw_stream(qw_model *m) { return m ? (void *)m->st : nullptr; }

int32_t qw_last_launch_count(const qw_model *m) { return m ? m->launches : 0; }

const char *qw_last_error(const qw_model *m) { return m ? m->err.c_str() : qw::op_last_error(); }

void qw_destroy(qw_model *m) {
    if (!m) return;
    cudaSetDevice(m->dev);
    if (m->st) cudaStreamSynchronize(m->st);
    if (m->graph) cudaGraphExecDestroy(m->graph);
    for (auto e : m->prof_ev) cudaEventDestroy(e);
    for (auto &Ly : m->L) {
        cudaFree(Ly.w_qkv); cudaFree(Ly.b_qkv); cudaFree(Ly.qn); cudaFree(Ly.kn); cudaFree(Ly.w_o);
        cudaFree(Ly.w_gu); cudaFree(Ly.w_down); cudaFree(Ly.rms_att); cudaFree(Ly.rms_ffn);
    }
    if (!m->lm_alias) cudaFree(m->lm);
    cudaFree(m->embed); cudaFree(m->norm_final); cudaFree(m->freq);
    cudaFree(m->kpool); cudaFree(m->vpool); cudaFree(m->d_page_table);
    cudaFree(m->xa); cudaFree(m->xb); cudaFree(m->part); cudaFree(m->qkv); cudaFree(m->attn); cudaFree(m->hbuf);
    cudaFree(m->part_o); cudaFree(m->part_ml); cudaFree(m->qk_ss); cudaFree(m->counters); cudaFree(m->am_counter);
    cudaFree(m->am_pval); cudaFree(m->am_pidx); cudaFree(m->am_val); cudaFree(m->am_idx); cudaFree(m->am_val_all);
    cudaFree(m->am_idx_all); cudaFree(m->logits); cudaFree(m->logits_all); cudaFree(m->d_tokens); cudaFree(m->d_argmax);
    cudaFree(m->d_step_layers); cudaFree(m->d_bar); cudaFree(m->gu); cudaFree(m->gu_split); cudaFree(m->qkv_split); cudaFree(m->part_split); cudaFree(m->cand_val); cudaFree(m->cand_idx); cudaFree(m->d_trace);
    for (void *q : m->xch_peer)
        if (q) cudaIpcCloseMemHandle(q);
    cudaFree(m->xch); cudaFree(m->d_xch); cudaFree(m->d_persist);
    cudaFree(m->ar_buf); cudaFree(m->d_ar); cudaFree(m->ar_ctr);
    cudaFree(m->d_rng); cudaFree(m->d_samp);
    if (m->h_pin_i) cudaFreeHost(m->h_pin_i);
    prefill_free(m->pf);
    if (m->comm) ncclCommDestroy(m->comm);
    if (m->st) cudaStreamDestroy(m->st);
    cudaGetLastError();  // a failed release leaves no error for the next call of this thread to report
    delete m;
}

}  // extern "C"

// qw_kernels.h -- host-side launch interface of the kernels in libqwen3_b200.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "qw_internal.cuh"

#define QW_STR2(x) #x
#define QW_STR(x) QW_STR2(x)

namespace qw {

struct PlaceArgs {
    void *dst;
    int dst_bf16;
    int dst_ld;
    int dst_row0;
    int row_map;  // 0 = dst_row0 + r, 1 = gate rows of the interleaved gate/up matrix, 2 = up rows
    int rows, cols;
    // source: host-copied slice ...
    const void *src;
    int src_dtype;  // 0 f32, 1 bf16, 2 f64
    int src_ld;
    // ... or the synthetic generator over the full tensor
    int synth;
    int constant_one;
    uint64_t seed;
    uint32_t tensor_id;
    float scale;
    int src_row0, src_col0;
    long long full_cols;
};

cudaError_t place_launch(const PlaceArgs &p, cudaStream_t st);
cudaError_t freq_launch(float2 *freq, int seq_len, int head_dim, double theta, cudaStream_t st);
cudaError_t argmax_merge_launch(const float *vals, const int *idxs, int tp, int B, int *argmax_out, int *next_tokens,
                                int *positions, int advance, int *hist, int hist_ld, cudaStream_t st);
cudaError_t qk_sumsq_launch(const float *qkv, int ld, int qw, int kw, int B, float *out, cudaStream_t st);
cudaError_t hold_launch(unsigned long long ns, cudaStream_t st);
cudaError_t add_launch(float *out, const float *a, const float *b, size_t n, cudaStream_t st);
cudaError_t zero_launch(float *out, size_t n, cudaStream_t st);  // programmatically launched; memset when unaligned
cudaError_t swiglu_rows_launch(float *gu, int T, int F, __nv_bfloat16 *h, cudaStream_t st);  // zeroes gu after reading

struct NormRowsArgs {
    float *x;  // (rows, ld_x) fp32 residual stream: read, or written when embed / part is given
    int ld_x;
    float *part;  // optional (rows, ld_part) all-reduced partial added to x (and stored)
    int ld_part;
    int zero_part;  // write zeros over the partial after reading it (the next split-K GEMM accumulates into it)
    const __nv_bfloat16 *embed;  // optional (vocab, K) bf16 table: x = embed[tokens[r]] (stored)
    const int *tokens;
    const float *w;  // rmsnorm weight (K)
    float eps;
    __nv_bfloat16 *out;  // (rows, ld_out) bf16 normalised rows
    int ld_out;
    int K;
};

struct QkvPostArgs {
    float *qkv;  // (rows, ld_qkv) fp32: q | k | v of this rank's heads
    int ld_qkv;
    int zero_qkv;  // write zeros over the rows read (the next split-K GEMM accumulates into them)
    const float *qn, *kn;
    int qk_mode;         // 0 none, 1 whole vector, 2 per head
    const float *qk_ss;  // optional (rows, 2) global sums of squares (vector mode, tp > 1)
    int q_total, kv_total;
    const float2 *freq;
    const int *slots, *positions;  // per row
    const int *page_table;
    int max_pages, page_size, log2_page;
    void *kcache, *vcache;  // this layer
    int H, Hkv, d;
    __nv_bfloat16 *q_out;  // (rows, ld_q) bf16 rotated queries
    int ld_q;
    // optional (vector mode, tp > 1, rows <= SM count): the sums of squares exchanged over NVLink inside the
    // kernel instead of qk_ss: flag-in-data words in every rank's inbox [rows][tp][2] at word offset xoff
    unsigned long long *const *xpeers;
    long long xoff;
    int tp, rank;
    unsigned *gen, *done;  // generation / CTA arrivals shared with the all-reduce kernels (qw_allreduce.cu)
    int *err;
};

struct FlashArgs {
    const __nv_bfloat16 *q;  // (nseq * L, ld_q): sequence b's rows b*L .. b*L+L-1
    int ld_q;
    const void *kcache, *vcache;  // this layer, bf16
    const int *page_table;
    int max_pages, page_size, log2_page;
    const int *seq_slots;  // (nseq)
    int p0, L;             // the chunk covers positions p0 .. p0+L-1 of every sequence
    int H, Hkv, d;
    float scale;
    __nv_bfloat16 *out;  // (nseq * L, ld_out)
    int ld_out;
    int num_pages;  // pages of the KV pool (the tensor-core kernel's TMA descriptor of the cache)
    int *err;       // device error word (bounded waits)
};

struct FlashDecodeArgs {
    const __nv_bfloat16 *q;  // (B, ld_q) rotated queries (this rank's heads)
    int ld_q;
    const void *kcache, *vcache;  // this layer, bf16; the current position already written
    const int *page_table;
    int max_pages, page_size, log2_page;
    const int *slots, *positions;  // (B)
    int H, Hkv, d;
    int nsplit;  // context splits (<= 64), merged by the last CTA of each (sequence, KV head)
    float scale;
    float *part_o, *part_ml;  // (B, H, nsplit, d), (B, H, nsplit, 2)
    unsigned *counters;       // (B, Hkv), zero on entry, reset on exit
    __nv_bfloat16 *out;       // (B, ld_out)
    int ld_out;
    int num_pages;            // pages of the KV pool (the TMA descriptors of the cache)
    int *err;                 // device error word (bounded waits)
};

struct RowsArgmaxArgs {
    const float *logits;  // (rows, ld)
    int ld, n;
    const float *cand_val;  // instead of logits: (rows, ld) candidate maxima with their indices (n per row)
    const int *cand_idx;
    int idx_offset;
    int *argmax_out;
    float *argmax_val;
    int *next_tokens, *positions;
    int advance;
    int *hist;
    int hist_ld;
};

struct SampleArgs {
    const float *logits;  // (rows, ld)
    int ld, V;
    double temperature;   // <= 0: greedy
    double top_p;         // mode 1 only; >= 1: no nucleus filter
    int mode;             // 0: the Qwen3 generation sampler (softmax, then sampleToken's second softmax); 1: sampleToken
    const double *r;      // (rows) uniform draws, or nullptr: draw from rng
    unsigned long long *rng;  // (rows) java.util.Random states
    double *scratch;      // (rows, V)
    int *out;             // (rows) nullable
    int *next_tokens, *positions;  // advance: next_tokens[row] = token, positions[row] += 1
    int advance;
    int *hist;
    int hist_ld;
};

cudaError_t sample_rows_launch(const SampleArgs &a, int rows, cudaStream_t st);
unsigned long long java_random_state(long long seed);

cudaError_t norm_rows_launch(const NormRowsArgs &a, int rows, cudaStream_t st);
cudaError_t qkv_post_launch(const QkvPostArgs &a, int rows, bool kv_bf16, cudaStream_t st);
cudaError_t flash_prefill_launch(const FlashArgs &a, int nseq, cudaStream_t st);
// head_dim 128 on tcgen05 (qw_attn_tc.cu); flash_prefill_tc_prepare opts it in to its shared memory
cudaError_t flash_prefill_tc_launch(const FlashArgs &a, int nseq, cudaStream_t st);
cudaError_t flash_prefill_tc_prepare();
cudaError_t rows_argmax_launch(const RowsArgmaxArgs &a, int rows, cudaStream_t st);
cudaError_t flash_decode_launch(const FlashDecodeArgs &a, int B, cudaStream_t st);
cudaError_t prefill_kernels_prepare();  // opt the row kernels in to their shared memory (once, before capture)

// ---- persistent batch-1 decode step (qw_step.cu) ----
struct StepLayer {
    const __nv_bfloat16 *w_qkv, *w_o, *w_gu, *w_down;
    const float *b_qkv, *qn, *kn, *rms_att, *rms_ffn;
    void *kc, *vc;  // this layer's KV pool
};

struct StepArgs {
    const StepLayer *L;  // device array (layers)
    int layers;
    int D, F, V, H, Hkv, d;  // hidden, intermediate, vocab, heads, KV heads, head_dim (tp = 1)
    const __nv_bfloat16 *embed, *lm;
    const float *norm_final;
    float eps, scale;
    int qk_mode;
    const float2 *freq;
    const int *page_table;
    int max_pages, page_size, log2_page;
    const int *slots;         // device scalar (nullable: slot 0)
    int *tokens, *positions;  // device scalars
    int advance;
    int *hist;
    int *argmax_out;
    float *logits;  // optional (V)
    float *x, *qkv, *attn, *gu;  // work vectors (D), (Q + 2 KV), (Q), (2 F)
    float *part_o, *part_ml;
    unsigned *counters;  // (layers, Hkv) attention split arrivals, zeroed before each launch
    float *am_val;         // (grid) per-CTA argmax candidates
    int *am_idx;
    unsigned *bar;         // grid barrier counter, zeroed before each launch
    float *ss;             // (layers, 2) q / k sums of squares, zeroed before each launch
    int *err;
    // tensor parallelism (tp = 1: none)
    int tp, rank, v0;          // ranks, this rank, first vocabulary row of this rank's lm_head shard
    int q_total, kv_total;     // global q / k widths (whole-vector QK-norm denominators)
    unsigned *const *xch;      // device array [tp]: every rank's exchange buffer (peer pointers)
    unsigned *gen;             // cross-rank barriers passed, persistent across steps
    int max_k, max_rows, xs_floats;  // shared-memory layout
    int stage_off;                   // floats: staged attention keys within the activation region
    int kv_bf16;
    unsigned long long *trace;       // optional: CTA 0's globaltimer before / after every grid barrier
    int evict_first;                 // weight stream marked L2 evict-first (keeps code, KV and activations resident)
    unsigned long long wait_cycles;  // bound of every wait in SM clock cycles; on expiry the kernel reports and returns
    int row_copies;                  // ring: one bulk copy per weight row (else one per slot when rows are contiguous)
    int stall_cta;                   // test hook (-1 = off): this CTA withholds its arrival at the step's first barrier
};

size_t step_smem_bytes(const StepArgs &a);
// Fills a.max_k / max_rows / xs_floats; false when the geometry or shared memory does not fit.
bool step_layout(StepArgs &a, int grid, size_t *smem_out);
cudaError_t step_prepare(bool kv_bf16, int d, int G, bool tp, size_t smem);
cudaError_t step_launch(const StepArgs &a, bool kv_bf16, int grid, cudaStream_t st);
const void *step_kernel_fn(bool kv_bf16, int d, int G, bool tp);
constexpr int kStepBlockThreads = 288;

cudaError_t gemv_launch(const GemvArgs &a, int epi, bool bf16, int num_sms, cudaStream_t st);
cudaError_t attn_decode_launch(const AttnArgs &a, int B, bool kv_bf16, cudaStream_t st);

}  // namespace qw

/*
 * qwen3_b200.h -- C ABI of libqwen3_b200.so, the B200 (sm_100a) backend for the
 * almostrealism/common Qwen3 forward step.
 *
 * The reference runs this step as a Java operation graph (engine/ml Qwen3 ->
 * CompiledModel) lowered to generated C kernels that are entered through JNI, one
 * kernel per graph node:
 *   JNIEXPORT void JNICALL Java_<GeneratedOperationN>_apply(JNIEnv*, jobject, jlong commandQueue,
 *       jlongArray arg, jintArray offset, jintArray size, jint count, jint globalId, jlong kernelSize)
 *   (base/hardware/src/main/resources/.../generated.javatemplate:21-25,
 *    base/hardware/src/main/java/org/almostrealism/hardware/jni/NativeInstructionSet.java:39-121)
 * This library replaces the whole compiled model rather than individual graph nodes:
 * one call runs the full forward step of every layer.  Each entry point below names
 * the reference call it stands in for.
 *
 * Conventions
 *   - plain C types only; every function returns qw_status (0 = OK);
 *   - host buffers are borrowed for the duration of the call, never retained;
 *   - the library owns all device memory it allocates;
 *   - calls on one qw_model must be serialised by the caller (the reference's
 *     AutoregressiveModel is single-threaded as well);
 *   - one CUDA stream per model; `*_device` entry points take device pointers and
 *     enqueue on that stream without synchronising.
 */
#ifndef QWEN3_B200_H
#define QWEN3_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QW_ABI_VERSION 1

typedef int32_t qw_status;
enum {
    QW_OK = 0,
    QW_ERR_ARG = 1,         /* null pointer / bad argument (reference: NullPointerException) */
    QW_ERR_SHAPE = 2,       /* tensor or batch shape mismatch (IllegalArgumentException) */
    QW_ERR_OOM = 3,         /* device allocation failed */
    QW_ERR_CUDA = 4,        /* CUDA runtime error */
    QW_ERR_NCCL = 5,        /* NCCL error */
    QW_ERR_TIMEOUT = 6,     /* a bounded device wait gave up */
    QW_ERR_STATE = 7,       /* call not valid in this state (e.g. weights not finalized) */
    QW_ERR_UNSUPPORTED = 8, /* configuration not supported by this build */
    QW_ERR_KEY = 9          /* unknown state-dict key */
};

typedef enum { QW_DTYPE_F32 = 0, QW_DTYPE_BF16 = 1, QW_DTYPE_F64 = 2 } qw_dtype;

/* QK-norm variants.  QW_QKNORM_VECTOR is the reference's behaviour: rmsnorm over the
 * whole projected q (and k) vector with the (heads, head_dim) weight flattened
 * (engine/ml/src/main/java/org/almostrealism/ml/AttentionFeatures.java:840-845, 886-891).
 * QW_QKNORM_HEAD normalises each head over head_dim (HuggingFace Qwen3). */
typedef enum { QW_QKNORM_NONE = 0, QW_QKNORM_VECTOR = 1, QW_QKNORM_HEAD = 2 } qw_qknorm;

/* Model geometry: engine/ml/src/main/java/org/almostrealism/ml/qwen3/Qwen3Config.java:574-588 and
 * TransformerConfig.java:94-105.  head_dim is explicit (the reference derives dim/heads,
 * TransformerConfig.java:104); heads*head_dim may differ from dim. */
typedef struct qw_config {
    int32_t dim;            /* hidden size */
    int32_t hidden_dim;     /* SwiGLU intermediate size */
    int32_t layers;
    int32_t heads;
    int32_t kv_heads;
    int32_t head_dim;       /* 64 or 128 */
    int32_t vocab;
    int32_t seq_len;        /* max positions per sequence slot (reference seqLen) */
    int32_t shared_weights; /* lm_head tied to model.embed_tokens.weight */
    int32_t qk_norm;        /* qw_qknorm */
    int32_t has_qkv_bias;   /* q/k/v projection biases (Qwen2.5 layout) */
    int32_t weight_dtype;   /* QW_DTYPE_F32 or QW_DTYPE_BF16: storage and GEMV input type */
    int32_t kv_dtype;       /* QW_DTYPE_F32 or QW_DTYPE_BF16 */
    int32_t max_batch;      /* sequence slots */
    int32_t max_tokens;     /* max tokens in one prefill call (activation arena), >= max_batch */
    int32_t page_size;      /* KV page size in tokens (power of two, 16..256); 0 = 64 */
    int32_t num_pages;      /* KV pages per rank; 0 = max_batch * ceil(seq_len / page_size) */
    int32_t decode_kernels; /* batch-1 decode with bf16 weights: 0 = auto (one persistent kernel per step when the
                               geometry fits it, at any tp: its cross-GPU all-reduces are flag-in-data stores
                               into the peers' memory over NVLink), 1 = one kernel per operation (+ NCCL under
                               tensor parallelism), 2 = the persistent kernel (as 0) */
    int32_t wait_limit_us;  /* bound of every device-side wait (grid and cross-GPU barriers, copies in flight,
                               split merges) in microseconds; 0 = 2 s.  A wait that runs out stops the kernel,
                               which records the site; qw_synchronize then returns QW_ERR_TIMEOUT */
    int32_t test_stall_cta; /* test hook, 0 = off: CTA (test_stall_cta - 1) of the persistent decode step
                               withholds its arrival at the step's first barrier, so that the other CTAs' bounded
                               waits run out (exercises the QW_ERR_TIMEOUT path without a GPU fault) */
    int32_t reserved[2];
    double rope_theta;      /* 1e6 for Qwen3 */
    double eps;             /* rmsnorm epsilon, 1e-6 for Qwen3 */
} qw_config;

typedef struct qw_model qw_model;

/* Library version / build information ("sm_100a", ABI version). */
int32_t qw_abi_version(void);
const char *qw_build_info(void);

/* NCCL unique id (128 bytes) for tensor-parallel creation; call on rank 0 and share. */
qw_status qw_get_unique_id(void *out128);

/* Create a model on `device`.  tp_size > 1 shards every layer Megatron-style over
 * tp_size ranks (one process per GPU) and joins the NCCL communicator named by
 * nccl_unique_id.  Stands in for the Qwen3 constructor
 * (engine/ml/src/main/java/org/almostrealism/ml/qwen3/Qwen3.java:249-255). */
qw_status qw_create(const qw_config *cfg, int32_t device, int32_t tp_rank, int32_t tp_size,
                    const void *nccl_unique_id, qw_model **out);

/* Copy one state-dict tensor (HF key, Qwen3.java:361-382) from host memory.  Besides the HF keys,
 * "rope.freq_cis" (seq_len, head_dim / 2, 2) replaces the RoPE table computed from rope_theta (Llama2
 * checkpoints carry theirs, engine/ml/src/main/java/org/almostrealism/ml/llama2/Llama2Weights.java).  The
 * rank keeps only its shard.  Accepts F32, BF16 or F64 host data and converts to the
 * configured storage type.  Stands in for StateDictionary.get
 * (engine/ml/src/main/java/org/almostrealism/ml/StateDictionary.java:119-150). */
qw_status qw_load_tensor(qw_model *m, const char *key, qw_dtype dtype, const int64_t *dims,
                         int32_t ndims, const void *host_ptr);

/* Load the reference's protobuf state dictionary: `path` is one CollectionLibraryData file or a
 * directory whose non-hidden regular files each hold one (read in name order), as
 * StateDictionary(weightsDirectory) does (engine/ml/src/main/java/org/almostrealism/ml/StateDictionary.java:119-150,
 * message types in engine/ml/src/main/proto/collections.proto).  Each entry is decoded as
 * CollectionEncoder.decode does (`data` doubles when present, else `data_32` floats; an entry without
 * dimensions is skipped) and passed to qw_load_tensor; keys this model does not use are skipped.  As in
 * StateDictionary.loadWeights, a file that cannot be parsed, or an entry whose value count does not match its
 * dimensions, ends that file with a warning (stderr and qw_last_error; the call still returns QW_OK) and
 * loading continues with the next file.  A known key whose shape does not fit the model returns its
 * qw_load_tensor error.  *loaded_out (may be NULL) receives the number of tensors loaded. */
qw_status qw_load_state_dict_pb(qw_model *m, const char *path, int32_t *loaded_out);

/* Fill every weight on the device from the counter-based synthetic generator
 * (seed, std); all rmsnorm / q_norm / k_norm weights are set to 1. */
qw_status qw_init_synthetic(qw_model *m, uint64_t seed, float std);

/* Validate that every required tensor is present and build fused layouts. */
qw_status qw_finalize_weights(qw_model *m);

/* Clear a sequence slot (-1 = all): frees its KV pages and zeroes its length.
 * Stands in for CompiledModel.reset / AutoregressiveModel.reset
 * (domain/graph/src/main/java/org/almostrealism/model/CompiledModel.java:218-220). */
qw_status qw_reset(qw_model *m, int32_t slot);

/* Make sure slot `slot` has KV pages for positions [0, n_positions). */
qw_status qw_reserve(qw_model *m, int32_t slot, int32_t n_positions);

/* One forward step for `batch` sequences, one token each: token[b] at position
 * positions[b] of slot slots[b] (slots may be NULL = 0..batch-1).  Writes logits
 * (batch x vocab, fp32, may be NULL) and the greedy token (first index of the max,
 * AggregationFeatures.java:111-121; may be NULL).  Stands in for
 * CompiledModel.forward + indexOfMax (CompiledModel.java:189-198,
 * engine/ml/src/main/java/org/almostrealism/ml/AutoregressiveModel.java:295-308, 412-420). */
qw_status qw_decode_step(qw_model *m, const int32_t *tokens, const int32_t *slots,
                         const int32_t *positions, int32_t batch, float *logits_out,
                         int32_t *argmax_out);

/* Same as qw_decode_step with an embedding row supplied instead of a token id:
 * x_in is (batch, dim) fp32 -- CompiledModel.forward((1, dim)) exactly. */
qw_status qw_forward_hidden(qw_model *m, const float *x_in, const int32_t *slots,
                            const int32_t *positions, int32_t batch, float *logits_out,
                            int32_t *argmax_out);

/* Process `batch` prompts of `seq_len` tokens each (tokens row-major batch x seq_len)
 * into slots (NULL = 0..batch-1) starting at position 0.  Writes the logits / greedy
 * token of each prompt's last position (either may be NULL).  The reference has no
 * batched prefill (it feeds prompt tokens one per forward, AutoregressiveModel.java:296-299);
 * results equal feeding the tokens one by one, within the bf16 tolerance. */
qw_status qw_prefill(qw_model *m, const int32_t *tokens, const int32_t *slots, int32_t batch,
                     int32_t seq_len, float *logits_out, int32_t *argmax_out);

/* Greedy autoregressive generation (AutoregressiveModel.next loop,
 * AutoregressiveModel.java:295-308): prompts (batch x prompt_len) are fed first,
 * then each step feeds the argmax of the previous step's logits.  tokens_out
 * (batch x steps) receives the token fed at every step (prompt tokens included),
 * i.e. what next() returns.  steps >= prompt_len. */
qw_status qw_generate(qw_model *m, const int32_t *prompts, int32_t batch, int32_t prompt_len,
                      int32_t steps, int32_t *tokens_out);

/* Sampling for qw_generate and qw_decode_sample (AutoregressiveModel.setTemperature,
 * engine/ml/src/main/java/org/almostrealism/ml/AutoregressiveModel.java:47-61).  temperature <= 0:
 * greedy (the default).  mode 0: the sampler Qwen3 generates with (AutoregressiveModel.of, :405-434:
 * softmax of logits / temperature, then sampleToken(probabilities, vocab, 1.0, 1.0, random), which
 * applies a second softmax); mode 1: sampleToken(logits, vocab, temperature, top_p, random) (:323-386,
 * nucleus filtering when top_p < 1).  Slot s draws from its own java.util.Random(seed + s) sequence
 * (the same 48-bit generator, so a Java caller seeding identically draws the same numbers). */
qw_status qw_set_sampling(qw_model *m, double temperature, double top_p, int64_t seed, int32_t mode);

/* One decode step like qw_decode_step, with the next token drawn by the model's sampling settings
 * (greedy when the temperature is 0) into tokens_out (batch).  Stands in for AutoregressiveModel.next
 * after the prompt (AutoregressiveModel.java:295-308). */
qw_status qw_decode_sample(qw_model *m, const int32_t *tokens, const int32_t *slots, const int32_t *positions,
                           int32_t batch, int32_t *tokens_out);

/* Device-resident variant of qw_decode_step for benchmarking and graph replay:
 * all pointers are device pointers; enqueued on the model's stream.  Pages must
 * already be reserved (qw_reserve).  If advance != 0 the kernel writes the argmax
 * into d_tokens and increments d_positions, so repeated calls run greedy decode
 * with no host involvement. */
qw_status qw_decode_step_device(qw_model *m, int32_t *d_tokens, const int32_t *d_slots,
                                int32_t *d_positions, int32_t batch, float *d_logits,
                                int32_t *d_argmax, int32_t advance);

/* Capture the device decode step for `batch` into a CUDA graph (replayed by
 * qw_replay_decode) -- pointers as for qw_decode_step_device. */
qw_status qw_capture_decode(qw_model *m, int32_t *d_tokens, const int32_t *d_slots,
                            int32_t *d_positions, int32_t batch, float *d_logits, int32_t *d_argmax);
qw_status qw_replay_decode(qw_model *m, int32_t times);

/* Kernel classes reported by qw_profile_decode. */
enum {
    QW_KERNEL_OTHER = 0,
    QW_KERNEL_QKV = 1,     /* rmsnorm + fused q/k/v projection */
    QW_KERNEL_ATTN = 2,    /* QK-norm + RoPE + KV write + paged attention */
    QW_KERNEL_O = 3,       /* o projection + residual */
    QW_KERNEL_GATE_UP = 4, /* rmsnorm + gate/up projection + SwiGLU */
    QW_KERNEL_DOWN = 5,    /* down projection + residual */
    QW_KERNEL_LM_HEAD = 6, /* final rmsnorm + lm_head + argmax */
    QW_KERNEL_STEP = 7     /* the whole batch-1 decode step in one persistent kernel */
};

/* Set the device-side token / position of sequences 0..batch-1 (slots 0..batch-1) used by
 * qw_profile_decode, reserving KV pages. */
qw_status qw_set_device_inputs(qw_model *m, const int32_t *tokens, const int32_t *positions, int32_t batch);

/* Run one eager decode step on the model's own device inputs (qw_set_device_inputs) with
 * CUDA events around every kernel launch; writes up to `cap` launch durations (ms) and
 * their QW_KERNEL_* classes, and the launch count to *n_out.  Does not advance positions. */
qw_status qw_profile_decode(qw_model *m, int32_t batch, float *ms_out, int32_t *kinds_out, int32_t cap,
                            int32_t *n_out);

/* qw_prefill of (batch, seq_len) host tokens with CUDA events around every kernel launch (tensor-core
 * path only); writes up to `cap` launch durations (ms) and their QW_KERNEL_* classes and the launch count
 * to *n_out.  Stands in for nothing in the reference (a measurement aid; the reference feeds prompts one
 * token per forward, AutoregressiveModel.java:296-299). */
qw_status qw_profile_prefill(qw_model *m, const int32_t *tokens, const int32_t *slots, int32_t batch, int32_t seq_len,
                             float *ms_out, int32_t *kinds_out, int32_t cap, int32_t *n_out);

/* Wait for all work on the model's stream; QW_ERR_TIMEOUT if a bounded device-side wait gave up
 * since the model was created (a peer rank that never arrived, for instance). */
qw_status qw_synchronize(qw_model *m);

/* The model's CUDA stream (cudaStream_t) for event timing by the caller. */
void *qw_stream(qw_model *m);

/* Number of kernel launches the last decode step / prefill enqueued. */
int32_t qw_last_launch_count(const qw_model *m);

/* ---------------------------------------------------------------------------------------
 * Op-level entry points: one fused kernel over caller-provided DEVICE buffers, enqueued on
 * `stream` (a cudaStream_t, NULL = legacy default stream) of the current device.
 * -------------------------------------------------------------------------------------- */

/* Greedy sampling tail of the step: logits = W . rmsnorm(x; norm_w, eps) for `batch` (1..4)
 * hidden rows x (batch, dim) fp32, W (vocab, dim) in w_dtype (F32 or BF16); writes the
 * logits (batch, vocab) fp32 when logits_out is not NULL and the first index of the maximum
 * per row to argmax_out (batch) int32.  Stands in for rmsnorm(final) + dense(wcls) +
 * indexOfMax (Qwen3.java:402-405, AggregationFeatures.java:111-121,
 * AutoregressiveModel.java:412-420).  Its cross-CTA scratch is allocated with cudaMalloc on
 * the first call per device and kept for the life of the process; every call on a device shares
 * it, so calls that overlap on the GPU (different streams, no ordering between them) race. */
qw_status qw_op_lm_head_argmax(const void *w, int32_t w_dtype, int32_t vocab, int32_t dim, const float *x,
                               const float *norm_w, double eps, int32_t batch, float *logits_out,
                               int32_t *argmax_out, void *stream);

/* Batched projection on the tensor cores (tcgen05/TMEM, TMA-fed): for bf16 W (n_out, k) and bf16 X
 * (t, k), both row-major, acc(t, f) = sum_j W(f, j) X(t, j) in fp32, then by `epi`:
 *   QW_LINEAR_STORE   out fp32 (t, n_out) = acc (+ bias[f] when bias is not NULL)
 *   QW_LINEAR_RESID   out fp32 (t, n_out) = resid (t, n_out) + acc  (out may equal resid)
 *   QW_LINEAR_SWIGLU  W rows interleaved in blocks of 16 gate rows then 16 up rows;
 *                     out bf16 (t, n_out/2) = up * silu(gate)
 * k a multiple of 8, pointers 16-byte aligned, n_out a multiple of 32 for SWIGLU.  Stands in
 * for LayerFeatures.dense applied to t rows (domain/graph/src/main/java/org/almostrealism/layers/
 * LayerFeatures.java:785-830) with SequentialBlock.accum (SequentialBlock.java:413-429) and the
 * SwiGLU product (engine/ml/src/main/java/org/almostrealism/ml/FeedForwardFeatures.java:147-156). */
enum { QW_LINEAR_STORE = 0, QW_LINEAR_RESID = 1, QW_LINEAR_SWIGLU = 2 };
qw_status qw_op_linear(const void *w, int32_t n_out, int32_t k, const void *x, int32_t t, int32_t epi,
                       const float *bias, const float *resid, void *out, void *stream);

/* Token sampling over caller-provided device buffers: rows of logits (rows, ld) fp32, one uniform draw
 * in [0, 1) per row (r_uniform, device), scratch (rows, vocab) doubles; tokens_out (rows) int32.
 * temperature <= 0 is the first-index argmax; mode as for qw_set_sampling.  Stands in for
 * AutoregressiveModel.sampleToken (AutoregressiveModel.java:323-386) and the sampler of
 * AutoregressiveModel.of (:405-434), given the random draw. */
qw_status qw_op_sample(const float *logits, int32_t rows, int32_t vocab, int32_t ld, double temperature, double top_p,
                       int32_t mode, const double *r_uniform, double *scratch, int32_t *tokens_out, void *stream);

/* qw_op_lm_head_argmax with no allocation anywhere: same arguments, results and errors,
 * but its cross-CTA scratch is a fixed 64 KiB array compiled into the library (held on every
 * GPU that loads it until the process exits) instead of memory from cudaMalloc.  For hosts
 * that cannot allocate device memory themselves or through this library -- a JVM that only
 * passes pointers into its own pool, a process whose caching allocator must own every byte.
 * No counterpart in the reference (its generated kernels never need scratch).
 * Limit: sm_count * 8 * batch <= 8192 (every current GPU at batch <= 4); beyond it the call
 * returns QW_ERR_SHAPE.  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call before any stream
 * capture.  All calls share the one array: calls that overlap on the GPU (other streams,
 * other host threads) race and must be serialised by the caller. */
qw_status qw_op_lm_head_argmax_static(const void *w, int32_t w_dtype, int32_t vocab, int32_t dim, const float *x,
                                      const float *norm_w, double eps, int32_t batch, float *logits_out,
                                      int32_t *argmax_out, void *stream);

/* Human-readable description of the last error on this model (never NULL).  With m == NULL:
 * the last error of an op-level entry point on this thread. */
const char *qw_last_error(const qw_model *m);

void qw_destroy(qw_model *m);

#ifdef __cplusplus
}
#endif
#endif

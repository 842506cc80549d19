// qw_ops.cu -- op-level entry points: single fused kernels over caller-provided device buffers.
//
// The reference enters its generated kernels one operation at a time through JNI
// (NativeInstructionSet.java:39-121); these entry points expose individual fused kernels of
// this library the same way, for hosts that keep their own device buffers.
#include <cuda_runtime.h>
#include <mutex>
#include <string>

#include "../../include/qwen3_b200.h"
#include "qw_kernels.h"
#include "qw_ops.h"
#include "qw_tc.h"

namespace qw {

static thread_local std::string g_op_error;

qw_status op_fail(qw_status s, const std::string &msg) {
    g_op_error = msg;
    return s;
}

const char *op_last_error() { return g_op_error.c_str(); }

qw_status op_lm_head_check(const void *w, int32_t w_dtype, int32_t vocab, int32_t dim, const float *x,
                           const float *norm_w, int32_t batch, const int32_t *argmax_out) {
    if (!w || !x || !norm_w || !argmax_out) return op_fail(QW_ERR_ARG, "null device pointer");
    if (w_dtype != QW_DTYPE_F32 && w_dtype != QW_DTYPE_BF16) return op_fail(QW_ERR_UNSUPPORTED, "weight dtype");
    if (vocab < 1 || dim < 8 || dim % 8) return op_fail(QW_ERR_SHAPE, "vocab >= 1 and dim a positive multiple of 8");
    if (batch < 1 || batch > kGemvMaxB) return op_fail(QW_ERR_SHAPE, "batch must be in [1, 4]");
    return QW_OK;
}

GemvArgs op_lm_head_args(const void *w, int32_t vocab, int32_t dim, const float *x, const float *norm_w, double eps,
                         int32_t batch, float *logits_out, int32_t *argmax_out, float *part_val, int *part_idx,
                         unsigned *counter) {
    GemvArgs g{};
    g.W = w; g.N = vocab; g.K = dim; g.B = batch;
    g.xin = x; g.ld_in = dim;
    g.norm_w = norm_w; g.eps = (float)eps;
    g.out = logits_out; g.ld_out = vocab;
    g.part_val = part_val; g.part_idx = part_idx; g.counter = counter;
    g.argmax_out = argmax_out;
    return g;
}

}  // namespace qw

using namespace qw;

namespace {
// per-device scratch of qw_op_lm_head_argmax, allocated on first use and kept
struct OpScratch {
    float *val = nullptr;
    int *idx = nullptr;
    unsigned *counter = nullptr;
};
std::mutex g_scratch_mu;
OpScratch g_scratch[64];
}  // namespace

extern "C" qw_status qw_op_lm_head_argmax(const void *w, int32_t w_dtype, int32_t vocab, int32_t dim, const float *x,
                                          const float *norm_w, double eps, int32_t batch, float *logits_out,
                                          int32_t *argmax_out, void *stream) {
    qw_status s = op_lm_head_check(w, w_dtype, vocab, dim, x, norm_w, batch, argmax_out);
    if (s) return s;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return op_fail(QW_ERR_CUDA, "no current device");
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return op_fail(QW_ERR_CUDA, "device query failed");
    cudaStream_t st = (cudaStream_t)stream;
    OpScratch *sc;
    {
        std::lock_guard<std::mutex> lk(g_scratch_mu);
        sc = &g_scratch[dev];
        if (!sc->val) {
            size_t n = (size_t)sms * kGemvMaxCtasPerSm * kGemvMaxB;
            if (cudaMalloc(&sc->val, n * sizeof(float)) != cudaSuccess ||
                cudaMalloc(&sc->idx, n * sizeof(int)) != cudaSuccess ||
                cudaMalloc(&sc->counter, sizeof(unsigned)) != cudaSuccess ||
                cudaMemset(sc->counter, 0, sizeof(unsigned)) != cudaSuccess) {
                cudaFree(sc->val); cudaFree(sc->idx); cudaFree(sc->counter);
                *sc = OpScratch{};
                return op_fail(QW_ERR_OOM, "scratch allocation failed");
            }
        }
    }
    GemvArgs g = op_lm_head_args(w, vocab, dim, x, norm_w, eps, batch, logits_out, argmax_out, sc->val, sc->idx,
                                 sc->counter);
    cudaError_t e = gemv_launch(g, EPI_ARGMAX, w_dtype == QW_DTYPE_BF16, sms, st);
    if (e != cudaSuccess) return op_fail(QW_ERR_CUDA, std::string("lm_head/argmax launch: ") + cudaGetErrorString(e));
    return QW_OK;
}

extern "C" qw_status qw_op_linear(const void *w, int32_t n_out, int32_t k, const void *x, int32_t t, int32_t epi,
                                  const float *bias, const float *resid, void *out, void *stream) {
    if (!w || !x || !out) return op_fail(QW_ERR_ARG, "null device pointer");
    if (epi < QW_LINEAR_STORE || epi > QW_LINEAR_SWIGLU) return op_fail(QW_ERR_ARG, "epilogue " + std::to_string(epi));
    if (epi == QW_LINEAR_RESID && !resid) return op_fail(QW_ERR_ARG, "RESID needs resid");
    if (n_out < 1 || t < 1 || k < 8 || k % 8) return op_fail(QW_ERR_SHAPE, "n_out, t >= 1 and k a positive multiple of 8");
    if (epi == QW_LINEAR_SWIGLU && n_out % 32) return op_fail(QW_ERR_SHAPE, "SWIGLU needs n_out a multiple of 32");
    if (((uintptr_t)w | (uintptr_t)x) & 15) return op_fail(QW_ERR_ARG, "w and x must be 16-byte aligned");
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return op_fail(QW_ERR_CUDA, "no current device");
    {
        static std::mutex mu;
        static bool prepared[64] = {};
        std::lock_guard<std::mutex> lk(mu);
        if (dev < 64 && !prepared[dev]) {
            cudaError_t e = tc_prepare();
            if (e != cudaSuccess) return op_fail(QW_ERR_CUDA, std::string("GEMM set-up: ") + cudaGetErrorString(e));
            prepared[dev] = true;
        }
    }
    TcArgs a{};
    a.M = n_out; a.T = t; a.K = k; a.ksplit = 1;
    a.out = out; a.ld_out = epi == QW_LINEAR_SWIGLU ? n_out / 2 : n_out;
    a.resid = resid; a.ld_resid = n_out; a.bias = epi == QW_LINEAR_STORE ? bias : nullptr;
    cudaError_t e = tc_gemm_launch(w, x, a, epi, 0, sms, (cudaStream_t)stream);
    if (e != cudaSuccess) return op_fail(QW_ERR_CUDA, std::string("linear launch: ") + cudaGetErrorString(e));
    return QW_OK;
}

extern "C" qw_status qw_op_sample(const float *logits, int32_t rows, int32_t vocab, int32_t ld, double temperature,
                                  double top_p, int32_t mode, const double *r_uniform, double *scratch,
                                  int32_t *tokens_out, void *stream) {
    if (!logits || !tokens_out || (temperature > 0.0 && (!r_uniform || !scratch)))
        return op_fail(QW_ERR_ARG, "null device pointer");
    if (rows < 1 || vocab < 1 || ld < vocab) return op_fail(QW_ERR_SHAPE, "rows, vocab >= 1 and ld >= vocab");
    if (mode != 0 && mode != 1) return op_fail(QW_ERR_ARG, "mode 0 or 1");
    if (!(top_p > 0.0)) return op_fail(QW_ERR_ARG, "top_p must be positive");
    SampleArgs a{};
    a.logits = logits; a.ld = ld; a.V = vocab; a.temperature = temperature; a.top_p = top_p; a.mode = mode;
    a.r = r_uniform; a.scratch = scratch; a.out = tokens_out;
    cudaError_t e = sample_rows_launch(a, rows, (cudaStream_t)stream);
    if (e != cudaSuccess) return op_fail(QW_ERR_CUDA, std::string("sample launch: ") + cudaGetErrorString(e));
    return QW_OK;
}

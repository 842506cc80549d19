// qw_noalloc.cu -- qw_op_lm_head_argmax_static: the fused rmsnorm + lm_head + argmax kernel
// with its cross-CTA scratch in a fixed device array instead of cudaMalloc'd memory.
//
// Some hosts cannot call cudaMalloc at all: a JVM that hands this library only memory it
// allocated itself through its own pool (the reference's Java side owns every buffer and
// passes borrowed pointers per call), a process whose CUDA allocations all go through a
// caching allocator that must see every byte, or code that runs while a stream is being
// captured, where an allocation is not allowed.  This entry point allocates nothing.
//
// The scratch (per-CTA partial maxima, their indices and the arrival counter) lives in
// file-scope __device__ arrays, so every GPU that loads the library holds
// kStaticSlots * 8 + 4 bytes (64 KiB + 4 B) until the process exits.
#include <cuda_runtime.h>
#include <mutex>
#include <string>

#include "../../include/qwen3_b200.h"
#include "qw_kernels.h"
#include "qw_ops.h"

using namespace qw;

namespace {

// (CTA, batch row) partial results the scratch holds: grid CTAs x batch must fit
constexpr int kStaticSlots = 8192;

static __device__ __align__(256) float g_static_val[kStaticSlots];
static __device__ __align__(256) int g_static_idx[kStaticSlots];
static __device__ __align__(256) unsigned g_static_counter[1];

// Device addresses of the arrays, looked up once per device.  The host-side names are
// stand-ins, not device addresses, so only these pointers are ever passed to a kernel.
struct StaticScratch {
    bool ready = false;
    float *val = nullptr;
    int *idx = nullptr;
    unsigned *counter = nullptr;
};
constexpr int kMaxDevices = 64;
std::mutex g_mu;
StaticScratch g_dev[kMaxDevices];

qw_status setup_device(int dev, StaticScratch **out) {
    std::lock_guard<std::mutex> lk(g_mu);
    StaticScratch &s = g_dev[dev];
    if (!s.ready) {
        cudaError_t e = cudaGetSymbolAddress((void **)&s.val, g_static_val);
        if (e == cudaSuccess) e = cudaGetSymbolAddress((void **)&s.idx, g_static_idx);
        if (e == cudaSuccess) e = cudaGetSymbolAddress((void **)&s.counter, g_static_counter);
        if (e != cudaSuccess)
            return op_fail(QW_ERR_CUDA, std::string("cudaGetSymbolAddress of the static scratch: ") +
                                            cudaGetErrorString(e));
        s.ready = true;
    }
    *out = &s;
    return QW_OK;
}

}  // namespace

extern "C" qw_status qw_op_lm_head_argmax_static(const void *w, int32_t w_dtype, int32_t vocab, int32_t dim,
                                                 const float *x, const float *norm_w, double eps, int32_t batch,
                                                 float *logits_out, int32_t *argmax_out, void *stream) {
    qw_status s = op_lm_head_check(w, w_dtype, vocab, dim, x, norm_w, batch, argmax_out);
    if (s) return s;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return op_fail(QW_ERR_CUDA, "no current device");
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return op_fail(QW_ERR_CUDA, "device query failed");
    // the GEMV grid is at most sms * kGemvMaxCtasPerSm CTAs, each writing `batch` partials
    long long need = (long long)sms * kGemvMaxCtasPerSm * batch;
    if (need > kStaticSlots)
        return op_fail(QW_ERR_SHAPE, "static scratch holds " + std::to_string(kStaticSlots) +
                                         " partial results; this device and batch need " + std::to_string(need));
    StaticScratch *sc = nullptr;
    s = setup_device(dev, &sc);
    if (s) return s;
    cudaStream_t st = (cudaStream_t)stream;
    // the arrival counter must start at zero; the kernel's last CTA resets it, this also
    // covers a previous call that did not finish
    cudaError_t e = cudaMemsetAsync(sc->counter, 0, sizeof(unsigned), st);
    if (e != cudaSuccess) return op_fail(QW_ERR_CUDA, std::string("counter reset: ") + cudaGetErrorString(e));
    GemvArgs g = op_lm_head_args(w, vocab, dim, x, norm_w, eps, batch, logits_out, argmax_out, sc->val, sc->idx,
                                 sc->counter);
    e = gemv_launch(g, EPI_ARGMAX, w_dtype == QW_DTYPE_BF16, sms, st);
    if (e != cudaSuccess) return op_fail(QW_ERR_CUDA, std::string("lm_head/argmax launch: ") + cudaGetErrorString(e));
    return QW_OK;
}

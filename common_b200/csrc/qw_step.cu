// qw_step.cu -- host side of the persistent batch-1 decode step (qw_step_impl.cuh): shared-memory layout,
// set-up and launch; instantiates the tp = 1 variants (the tensor-parallel ones are in qw_step_tp.cu, so the
// two compile in parallel).
#include "qw_step_impl.cuh"

namespace qw {

const void *step_fn_tp(bool kv_bf16, int d, int G);  // qw_step_tp.cu

namespace {
const void *step_fn(bool kv_bf16, int d, int G, bool tp) {
    if (tp) return step_fn_tp(kv_bf16, d, G);
    if (d == 128) return kv_bf16 ? step_fn_g<__nv_bfloat16, 128, false>(G) : step_fn_g<float, 128, false>(G);
    if (d == 64) return kv_bf16 ? step_fn_g<__nv_bfloat16, 64, false>(G) : step_fn_g<float, 64, false>(G);
    return nullptr;
}
}  // namespace

// q | k | v | 4 warp partials | 8 x (max, sum) | split (max, sum) | merge slice accumulators (<= G d)
static size_t attn_floats(int d, int G) { return (size_t)(G * d + 2 * d + 4 * G * d + 16 * G + 2 * G * 64 + G * d + 4); }

size_t step_smem_bytes(const StepArgs &a) {
    return (size_t)kRing * kPiece + (size_t)(a.xs_floats + a.max_rows) * sizeof(float);
}

bool step_layout(StepArgs &a, int grid, size_t *smem_out) {
    const int Q = a.H * a.d, KVw = a.Hkv * a.d, G = a.H / a.Hkv;
    if (a.D % 512 || Q % 512 || a.F % 512) return false;
    if (a.d != 64 && a.d != 128) return false;
    if (G < 1 || G > 8 || G == 3 || G == 5) return false;
    a.max_k = std::max(a.D, std::max(Q, a.F));
    // staged keys sit above both the QKV phase's activation vector and the attention scratch
    a.stage_off = (int)((std::max((size_t)a.D, attn_floats(a.d, G)) + 31) & ~(size_t)31);
    const size_t stage_bytes = (size_t)2 * a.d * (a.kv_bf16 ? 2 * stage_keys<__nv_bfloat16>() : 4 * stage_keys<float>());
    a.xs_floats = (int)std::max((size_t)a.max_k, (size_t)a.stage_off + stage_bytes / 4);
    a.xs_floats = (a.xs_floats + 3) & ~3;
    const int maxn = std::max(std::max(Q + 2 * KVw, 2 * a.F), std::max(a.D, a.V));
    a.max_rows = (maxn + grid - 1) / grid + 1;
    const size_t smem = step_smem_bytes(a);
    if (smem_out) *smem_out = smem;
    return smem + 4096 <= 227 * 1024;
}

const void *step_kernel_fn(bool kv_bf16, int d, int G, bool tp) { return step_fn(kv_bf16, d, G, tp); }

cudaError_t step_prepare(bool kv_bf16, int d, int G, bool tp, size_t smem) {
    const void *fn = step_fn(kv_bf16, d, G, tp);
    if (!fn) return cudaErrorInvalidValue;
    return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

cudaError_t step_launch(const StepArgs &a, bool kv_bf16, int grid, cudaStream_t st) {
    const void *fn = step_fn(kv_bf16, a.d, a.H / a.Hkv, a.tp > 1);
    if (!fn) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kStepThreads);
    cfg.dynamicSmemBytes = step_smem_bytes(a);
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    void *args[] = {const_cast<StepArgs *>(&a)};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace qw

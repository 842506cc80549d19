// qw_step_tp.cu -- the tensor-parallel (tp > 1) variants of the persistent decode step kernel.
#include "qw_step_impl.cuh"

namespace qw {

const void *step_fn_tp(bool kv_bf16, int d, int G) {
    if (d == 128) return kv_bf16 ? step_fn_g<__nv_bfloat16, 128, true>(G) : step_fn_g<float, 128, true>(G);
    if (d == 64) return kv_bf16 ? step_fn_g<__nv_bfloat16, 64, true>(G) : step_fn_g<float, 64, true>(G);
    return nullptr;
}

}  // namespace qw

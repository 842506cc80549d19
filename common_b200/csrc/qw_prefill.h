// qw_prefill.h -- buffers of the batched (prefill / large-batch) path.
#pragma once
#include <cuda_runtime.h>
#include "../../include/qwen3_b200.h"

namespace qw {

struct PrefillBuffers {
    float *x_host_stage = nullptr;  // (T, D) staging for host-supplied hidden rows
};

inline qw_status prefill_alloc(PrefillBuffers &pf, const qw_config &c, int T, int B, int Ql, int KVl, int Fl, int D) {
    (void)c; (void)B; (void)Ql; (void)KVl; (void)Fl;
    if (cudaMalloc((void **)&pf.x_host_stage, sizeof(float) * (size_t)T * D) != cudaSuccess) return QW_ERR_OOM;
    return QW_OK;
}

inline void prefill_free(PrefillBuffers &pf) {
    cudaFree(pf.x_host_stage);
    pf = PrefillBuffers{};
}

}  // namespace qw

// qw_prefill.h -- buffers of the batched (prefill / large-batch decode) path on the tensor cores.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include "../../include/qwen3_b200.h"

namespace qw {

struct PrefillBuffers {
    float *x_host_stage = nullptr;  // (T, D) staging for host-supplied hidden rows
    bool tc = false;                // tensor-core path available (bf16 weights and bf16 KV cache)
    __nv_bfloat16 *act = nullptr;   // (T, max(D, Ql)) normalised rows / attention output (GEMM operand)
    __nv_bfloat16 *q = nullptr;     // (T, Ql) rotated queries
    __nv_bfloat16 *h = nullptr;     // (T, Fl) SwiGLU output (GEMM operand)
    int *row_slot = nullptr, *row_pos = nullptr, *row_tok = nullptr;  // (T) per token row
    int *seq_slots = nullptr;       // (max_batch)
    float *row_ss = nullptr;        // (T, 2) global q/k sums of squares (vector QK-norm, tp > 1)
    int *h_pin = nullptr;           // pinned staging: row slots | row positions | row tokens | sequence slots
    int *d_err = nullptr;           // device error word of the tensor-core kernels
};

inline qw_status prefill_alloc(PrefillBuffers &pf, const qw_config &c, int T, int B, int Ql, int KVl, int Fl, int D) {
    (void)KVl;
    if (cudaMalloc((void **)&pf.x_host_stage, sizeof(float) * (size_t)T * D) != cudaSuccess) return QW_ERR_OOM;
    if (cudaMalloc((void **)&pf.d_err, sizeof(int)) != cudaSuccess) return QW_ERR_OOM;
    if (cudaMemset(pf.d_err, 0, sizeof(int)) != cudaSuccess) return QW_ERR_CUDA;
    pf.tc = c.weight_dtype == QW_DTYPE_BF16 && c.kv_dtype == QW_DTYPE_BF16;
    if (!pf.tc) return QW_OK;
    const size_t aw = (size_t)(D > Ql ? D : Ql);
    if (cudaMalloc((void **)&pf.act, sizeof(__nv_bfloat16) * (size_t)T * aw) != cudaSuccess ||
        cudaMalloc((void **)&pf.q, sizeof(__nv_bfloat16) * (size_t)T * Ql) != cudaSuccess ||
        cudaMalloc((void **)&pf.h, sizeof(__nv_bfloat16) * (size_t)T * Fl) != cudaSuccess ||
        cudaMalloc((void **)&pf.row_slot, sizeof(int) * (size_t)(3 * T + B)) != cudaSuccess ||
        cudaMalloc((void **)&pf.row_ss, sizeof(float) * (size_t)2 * T) != cudaSuccess)
        return QW_ERR_OOM;
    pf.row_pos = pf.row_slot + T;
    pf.row_tok = pf.row_pos + T;
    pf.seq_slots = pf.row_tok + T;
    if (cudaHostAlloc((void **)&pf.h_pin, sizeof(int) * (size_t)(3 * T + B), cudaHostAllocDefault) != cudaSuccess)
        return QW_ERR_OOM;
    return QW_OK;
}

inline void prefill_free(PrefillBuffers &pf) {
    cudaFree(pf.x_host_stage);
    cudaFree(pf.d_err);
    cudaFree(pf.act);
    cudaFree(pf.q);
    cudaFree(pf.h);
    cudaFree(pf.row_slot);
    cudaFree(pf.row_ss);
    if (pf.h_pin) cudaFreeHost(pf.h_pin);
    pf = PrefillBuffers{};
}

}  // namespace qw

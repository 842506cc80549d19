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

cudaError_t gemv_launch(const GemvArgs &a, int epi, bool bf16, int num_sms, cudaStream_t st);
cudaError_t attn_decode_launch(const AttnArgs &a, int B, bool kv_bf16, cudaStream_t st);

}  // namespace qw

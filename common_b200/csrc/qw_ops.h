// qw_ops.h -- shared helpers of the op-level entry points.
#pragma once
#include <string>
#include "../../include/qwen3_b200.h"
#include "qw_internal.cuh"

namespace qw {

// upper bound of resident 256-thread GEMV CTAs per SM (2048 threads / 256)
constexpr int kGemvMaxCtasPerSm = 8;

qw_status op_fail(qw_status s, const std::string &msg);
const char *op_last_error();
qw_status op_lm_head_check(const void *w, int32_t w_dtype, int32_t vocab, int32_t dim, const float *x,
                           const float *norm_w, int32_t batch, const int32_t *argmax_out);
GemvArgs op_lm_head_args(const void *w, int32_t vocab, int32_t dim, const float *x, const float *norm_w, double eps,
                         int32_t batch, float *logits_out, int32_t *argmax_out, float *part_val, int *part_idx,
                         unsigned *counter);

}  // namespace qw

// qw_ar.h -- host interface of the NVLink flag-in-data all-reduce (qw_allreduce.cu).
#pragma once
#include <cuda_runtime.h>

namespace qw {

struct ArArgs {
    float *x;                            // (n) this rank's partial, replaced by the sum over the ranks
    long long n;
    int tp, rank;
    unsigned long long *const *peers;    // device array [tp]: every rank's inbox ([tp][chunk] scatter | [n] gather)
    long long gather_off;                // words: offset of the gather inbox (tp * chunk)
    unsigned *gen;                       // device: generation of the last call (advanced by the kernel)
    unsigned *done;                      // device: CTA arrival counter, zero between calls
    int *err;                            // device error word: 6 when a wait ran out
};

// Inbox words one rank needs for an all-reduce of up to n elements over tp ranks.
inline long long allreduce_ll_words(long long n, int tp) { return (long long)tp * ((n + tp - 1) / tp) + n; }

cudaError_t allreduce_ll_launch(const ArArgs &a, int num_sms, cudaStream_t st);

}  // namespace qw

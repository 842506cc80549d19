// qw_ar.h -- host interface of the NVLink flag-in-data all-reduce (qw_allreduce.cu).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>

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

// The all-reduce of one row block fused with what follows it in the decode step: x += sum over the ranks of part
// (the residual accumulation after O or down), then rmsnorm(x) * w -> out (bf16, the next projection's operand).
// One CTA per row; the row's columns are owned in tp contiguous chunks (D / tp each): scatter to the owners, the
// owner adds the tp words in rank order and gathers the sum to every rank, every rank finishes the row.
struct ArNormArgs {
    float *part;      // (rows, ld_part) this rank's partial; zeroed after it is read when zero_part
    int ld_part, zero_part;
    float *x;         // (rows, D) residual stream, updated in place
    const float *w;   // (D) rmsnorm weight
    float eps;
    __nv_bfloat16 *out;  // (rows, ld_out)
    int ld_out, D, rows;
    int tp, rank;
    unsigned long long *const *peers;  // every rank's inbox: scatter [tp][rows][D / tp] | gather [rows][D]
    unsigned *gen, *done;
    int *err;
};
// D a multiple of 4 * tp, rows <= the SM count (every CTA of every rank resident at once)
cudaError_t ar_norm_launch(const ArNormArgs &a, int num_sms, cudaStream_t st);

#ifdef __CUDACC__
// 8-byte flag-in-data words over NVLink: fp32 value | generation << 32, one 64-bit store, single-copy atomic
__device__ __forceinline__ void xw_store(unsigned long long *p, float v, unsigned gen) {
    const unsigned long long w = (unsigned long long)__float_as_uint(v) | ((unsigned long long)gen << 32);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long xw_load(const unsigned long long *p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
// two adjacent words (16-byte aligned): one 16-byte access, each 8-byte half single-copy atomic on its own
__device__ __forceinline__ void xw_store2(unsigned long long *p, float v0, float v1, unsigned gen) {
    const unsigned long long w0 = (unsigned long long)__float_as_uint(v0) | ((unsigned long long)gen << 32);
    const unsigned long long w1 = (unsigned long long)__float_as_uint(v1) | ((unsigned long long)gen << 32);
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(w0), "l"(w1) : "memory");
}
__device__ __forceinline__ void xw_load2(const unsigned long long *p, unsigned long long &w0, unsigned long long &w1) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(p) : "memory");
}
// a word already loaded into w: spin (bounded) until it shows gen, then its value
__device__ __forceinline__ bool xw_settle(const unsigned long long *p, unsigned long long w, unsigned gen, float &v,
                                          unsigned long long limit) {
    if ((unsigned)(w >> 32) != gen) {
        const unsigned long long t0 = clock64();
        do {
            if ((unsigned long long)clock64() - t0 > limit) return false;
            w = xw_load(p);
        } while ((unsigned)(w >> 32) != gen);
    }
    v = __uint_as_float((unsigned)w);
    return true;
}
// bounded wait (limit in SM cycles) for the word at p to show generation gen; false on expiry
__device__ __forceinline__ bool xw_wait(const unsigned long long *p, unsigned gen, float &v,
                                        unsigned long long limit) {
    unsigned long long w = xw_load(p);
    if ((unsigned)(w >> 32) != gen) {
        const unsigned long long t0 = clock64();
        do {
            if ((unsigned long long)clock64() - t0 > limit) return false;
            w = xw_load(p);
        } while ((unsigned)(w >> 32) != gen);
    }
    v = __uint_as_float((unsigned)w);
    return true;
}
#endif

}  // namespace qw

// qw_allreduce.cu -- the all-reduce of the batched tensor-parallel decode step (the fp32 partials after the O
// and down projections, AttentionFeatures.java:922 and FeedForwardFeatures.java:154, and the QK-norm sums of
// squares) as one kernel over NVLink peer memory, in two shots:
//   1. reduce-scatter: element i belongs to chunk c = i / chunk, owned by rank c; every rank stores its partial
//      of i into slot `rank` of rank c's scatter inbox;
//   2. the owner waits for the tp words of each of its elements, adds them in rank order (every rank gets the same
//      sum) and stores the sum into every rank's gather inbox;
//   3. every rank waits for the gathered word of each element and writes it back over its partial.
// Every word is 8 bytes, fp32 value | generation << 32, written with one 64-bit store: a word showing this
// call's generation carries this call's value, so there is no barrier, no fence and no atomic on the data path.
// The generation is a device counter: all CTAs read it at entry, the last CTA to finish advances it (so the
// kernel can be captured in a CUDA graph).  Waits are bounded; on expiry the kernel records QW's timeout code.
#include <cuda_runtime.h>
#include <stdint.h>

#include "qw_internal.cuh"
#include "qw_ar.h"

namespace qw {

namespace {

constexpr int kArThreads = 512;
constexpr unsigned long long kArWaitCycles = 4000ull * 1000ull * 1000ull;  // ~2 s at 2 GHz

__device__ __forceinline__ void st_word(unsigned long long *p, float v, unsigned gen) {
    const unsigned long long w = (unsigned long long)__float_as_uint(v) | ((unsigned long long)gen << 32);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_word(const unsigned long long *p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
// bounded wait for the word at p to show generation gen; false on expiry
__device__ __forceinline__ bool wait_word(const unsigned long long *p, unsigned gen, float &v) {
    unsigned long long w = ld_word(p);
    if ((unsigned)(w >> 32) != gen) {
        const unsigned long long t0 = clock64();
        do {
            if ((unsigned long long)clock64() - t0 > kArWaitCycles) return false;
            w = ld_word(p);
        } while ((unsigned)(w >> 32) != gen);
    }
    v = __uint_as_float((unsigned)w);
    return true;
}

__global__ void __launch_bounds__(kArThreads) qw_allreduce_ll_kernel(ArArgs a) {
    griddep_wait();  // the partials come from the previous kernel
    __shared__ unsigned gen_sh;
    if (threadIdx.x == 0) gen_sh = *reinterpret_cast<volatile unsigned *>(a.gen) + 1u;
    __syncthreads();
    const unsigned gen = gen_sh;
    const long long n = a.n, chunk = (n + a.tp - 1) / a.tp;
    const long long nthr = (long long)gridDim.x * blockDim.x, t0 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    bool ok = true;
    // 1. scatter every element to its owner
    for (long long i = t0; i < n; i += nthr) {
        const int c = (int)(i / chunk);
        st_word(a.peers[c] + (size_t)a.rank * chunk + (i - (long long)c * chunk), a.x[i], gen);
    }
    // 2. reduce this rank's chunk, gather it to every rank
    const long long c0 = (long long)a.rank * chunk, c1 = c0 + chunk < n ? c0 + chunk : n;
    const unsigned long long *scat = a.peers[a.rank];
    for (long long i = c0 + t0; i < c1 && ok; i += nthr) {
        float s = 0.f;
        for (int p = 0; p < a.tp && ok; p++) {
            float v = 0.f;
            ok = wait_word(scat + (size_t)p * chunk + (i - c0), gen, v);
            s += v;
        }
        for (int p = 0; p < a.tp; p++) st_word(a.peers[p] + a.gather_off + i, s, gen);
    }
    // 3. every element's sum, back over the partial
    const unsigned long long *gath = a.peers[a.rank] + a.gather_off;
    for (long long i = t0; i < n && ok; i += nthr) {
        float v = 0.f;
        ok = wait_word(gath + i, gen, v);
        a.x[i] = v;
    }
    if (!ok && a.err) atomicExch(a.err, 6);
    // the last CTA advances the generation (every CTA has read it)
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(a.done, 1u) == gridDim.x - 1) {
            *a.done = 0u;
            *a.gen = gen;
        }
    }
    griddep_launch_dependents();
}

}  // namespace

cudaError_t allreduce_ll_launch(const ArArgs &a, int num_sms, cudaStream_t st) {
    if (a.n < 1 || a.tp < 2) return cudaErrorInvalidValue;
    long long blocks = (a.n + kArThreads - 1) / kArThreads;
    if (blocks > num_sms) blocks = num_sms;
    if (blocks < 1) blocks = 1;
    return launch_pdl(qw_allreduce_ll_kernel, dim3((unsigned)blocks), dim3(kArThreads), 0, st, a);
}

}  // namespace qw

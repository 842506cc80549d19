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

__device__ __forceinline__ void st_word(unsigned long long *p, float v, unsigned gen) { xw_store(p, v, gen); }
__device__ __forceinline__ bool wait_word(const unsigned long long *p, unsigned gen, float &v) {
    return xw_wait(p, gen, v, kArWaitCycles);
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

constexpr int kArNormThreads = 512;
constexpr int kArMaxTp = 8;

__global__ void __launch_bounds__(kArNormThreads) qw_ar_norm_kernel(ArNormArgs a) {
    griddep_wait();  // the partials come from the previous kernel
    extern __shared__ __align__(16) float xrow[];
    __shared__ float red[kArNormThreads / 32];
    __shared__ unsigned gen_sh;
    if (threadIdx.x == 0) gen_sh = *reinterpret_cast<volatile unsigned *>(a.gen) + 1u;
    __syncthreads();
    const unsigned gen = gen_sh;
    const int r = blockIdx.x, tid = threadIdx.x, D = a.D, cw = D / a.tp;
    float *prow = a.part + (size_t)r * a.ld_part;
    bool ok = true;
    // 1. scatter: column i of this row to its owner, rank i / cw (16-byte stores of two words)
    for (int i = tid * 4; i < D; i += kArNormThreads * 4) {
        const float4 v = *reinterpret_cast<const float4 *>(prow + i);
        if (a.zero_part) *reinterpret_cast<float4 *>(prow + i) = make_float4(0.f, 0.f, 0.f, 0.f);
        const int c = i / cw;
        unsigned long long *dst = a.peers[c] + ((size_t)a.rank * a.rows + r) * cw + (i - c * cw);
        xw_store2(dst, v.x, v.y, gen);
        xw_store2(dst + 2, v.z, v.w, gen);
    }
    // 2. this rank's columns, two at a time: every rank's words loaded at once (one round trip), added in rank
    //    order (the same sum on every rank), the sums stored to every rank
    const unsigned long long *scat = a.peers[a.rank];
    const size_t goff = (size_t)a.tp * a.rows * cw + (size_t)r * D + (size_t)a.rank * cw;
    for (int j = tid * 2; j < cw && ok; j += kArNormThreads * 2) {
        unsigned long long w[kArMaxTp][2];
#pragma unroll
        for (int p = 0; p < kArMaxTp; p++)
            if (p < a.tp) xw_load2(scat + ((size_t)p * a.rows + r) * cw + j, w[p][0], w[p][1]);
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int p = 0; p < kArMaxTp; p++)
            if (p < a.tp && ok) {
                const unsigned long long *src = scat + ((size_t)p * a.rows + r) * cw + j;
                float v0 = 0.f, v1 = 0.f;
                ok = xw_settle(src, w[p][0], gen, v0, kArWaitCycles) && xw_settle(src + 1, w[p][1], gen, v1, kArWaitCycles);
                s0 += v0;
                s1 += v1;
            }
        for (int p = 0; p < a.tp; p++) xw_store2(a.peers[p] + goff + j, s0, s1, gen);
    }
    // 3. the whole row: residual update, sum of squares (the gathered words of a round loaded at once)
    const unsigned long long *gath = a.peers[a.rank] + (size_t)a.tp * a.rows * cw + (size_t)r * D;
    float *xr = a.x + (size_t)r * D;
    float ss = 0.f;
    constexpr int kRound = 4;  // pairs in flight per thread
    for (int base = tid * 2; base < D && ok; base += kArNormThreads * 2 * kRound) {
        unsigned long long w[kRound][2];
#pragma unroll
        for (int u = 0; u < kRound; u++) {
            const int i = base + u * kArNormThreads * 2;
            if (i < D) xw_load2(gath + i, w[u][0], w[u][1]);
        }
#pragma unroll
        for (int u = 0; u < kRound; u++) {
            const int i = base + u * kArNormThreads * 2;
            if (i < D && ok) {
                float v0 = 0.f, v1 = 0.f;
                ok = xw_settle(gath + i, w[u][0], gen, v0, kArWaitCycles) &&
                     xw_settle(gath + i + 1, w[u][1], gen, v1, kArWaitCycles);
                const float2 xo = *reinterpret_cast<const float2 *>(xr + i);
                const float y0 = xo.x + v0, y1 = xo.y + v1;
                *reinterpret_cast<float2 *>(xr + i) = make_float2(y0, y1);
                *reinterpret_cast<float2 *>(xrow + i) = make_float2(y0, y1);
                ss += y0 * y0 + y1 * y1;
            }
        }
    }
    if (!ok && a.err) atomicExch(a.err, 6);
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kArNormThreads / 32; w++) tot += red[w];
    const float sc = 1.0f / sqrtf(tot / (float)D + a.eps);
    for (int k = tid * 4; k < D; k += kArNormThreads * 4) {
        const float4 v = *reinterpret_cast<const float4 *>(xrow + k);
        const float4 w = *reinterpret_cast<const float4 *>(a.w + k);
        uint2 o;
        o.x = (uint32_t)f2bf_bits(w.x * v.x * sc) | ((uint32_t)f2bf_bits(w.y * v.y * sc) << 16);
        o.y = (uint32_t)f2bf_bits(w.z * v.z * sc) | ((uint32_t)f2bf_bits(w.w * v.w * sc) << 16);
        *reinterpret_cast<uint2 *>(a.out + (size_t)r * a.ld_out + k) = o;
    }
    // the last CTA advances the generation (every CTA has read it)
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(a.done, 1u) == gridDim.x - 1) {
            *a.done = 0u;
            *a.gen = gen;
        }
    }
    // triggered last: an early trigger (the next GEMM streaming weights during the exchange) measured no faster
    griddep_launch_dependents();
}

}  // namespace

cudaError_t ar_norm_launch(const ArNormArgs &a, int num_sms, cudaStream_t st) {
    if (a.rows < 1 || a.rows > num_sms || a.tp < 2 || a.tp > kArMaxTp || a.D % (4 * a.tp) || a.D * sizeof(float) > 48 * 1024)
        return cudaErrorInvalidValue;
    return launch_pdl(qw_ar_norm_kernel, dim3((unsigned)a.rows), dim3(kArNormThreads), sizeof(float) * a.D, st, a);
}

cudaError_t allreduce_ll_launch(const ArArgs &a, int num_sms, cudaStream_t st) {
    if (a.n < 1 || a.tp < 2) return cudaErrorInvalidValue;
    long long blocks = (a.n + kArThreads - 1) / kArThreads;
    if (blocks > num_sms) blocks = num_sms;
    if (blocks < 1) blocks = 1;
    return launch_pdl(qw_allreduce_ll_kernel, dim3((unsigned)blocks), dim3(kArThreads), 0, st, a);
}

}  // namespace qw

// qw_sample.cu -- temperature / nucleus sampling of the next token on the device.
//
// Two behaviours of the reference (engine/ml/src/main/java/org/almostrealism/ml/AutoregressiveModel.java):
//   mode 0  the sampler Qwen3 generates with (AutoregressiveModel.of, :405-434): logits / temperature,
//           softmax, then sampleToken(probabilities, vocab, 1.0, 1.0, random) -- which applies a second
//           softmax to the probabilities -- and a categorical draw;
//   mode 1  sampleToken(logits, vocab, temperature, topP, random) itself (:323-386): softmax of
//           logits / temperature, nucleus filtering (descending probability, ties in index order, first
//           prefix whose cumulative probability reaches topP, renormalised), categorical draw.
// temperature <= 0 is the greedy first-index argmax in both.  The draw walks the probabilities in index
// order and returns the first index whose cumulative probability exceeds r (vocab - 1 if none), r from
// the caller or from a per-row java.util.Random state (the published 48-bit linear congruential
// generator: seed' = seed * 0x5DEECE66D + 0xB mod 2^48, nextDouble = (next(26) << 27 | next(27)) / 2^53).
// Arithmetic is double, as in the reference.  One CTA of 1024 threads per row; the nucleus cutoff is
// found by a radix select over the bit patterns of the (non-negative) probabilities, 6 histogram passes.
#include "qw_internal.cuh"
#include "qw_kernels.h"
#include <float.h>
#include <limits.h>

namespace qw {

namespace {

constexpr int kSampThreads = 1024;
constexpr int kSampWarps = kSampThreads / 32;

__device__ __forceinline__ double block_sum_d(double v, double *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double s = 0.0;
    for (int w = 0; w < kSampWarps; w++) s += red[w];
    return s;
}

__device__ __forceinline__ double block_max_d(double v, double *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double s = -DBL_MAX;
    for (int w = 0; w < kSampWarps; w++) s = fmax(s, red[w]);
    return s;
}

// java.util.Random: next(bits) on a scrambled 48-bit state
__device__ __forceinline__ int jr_next(unsigned long long &seed, int bits) {
    seed = (seed * 0x5DEECE66DULL + 0xBULL) & ((1ULL << 48) - 1);
    return (int)(seed >> (48 - bits));
}
__device__ __forceinline__ double jr_next_double(unsigned long long &seed) {
    const long long hi = (long long)jr_next(seed, 26);
    const long long lo = (long long)jr_next(seed, 27);
    return (double)((hi << 27) + lo) * (1.0 / 9007199254740992.0);
}

__global__ void __launch_bounds__(kSampThreads) qw_sample_rows_kernel(SampleArgs a) {
    __shared__ double red[kSampWarps];
    __shared__ double hist_m[2048];
    __shared__ int s_pick;
    __shared__ double s_r;
    __shared__ unsigned long long s_sel, s_cum;
    const int row = blockIdx.x, tid = threadIdx.x;
    const float *lg = a.logits + (size_t)row * a.ld;
    double *q = a.scratch + (size_t)row * a.V;
    const int V = a.V;
    int token;

    if (a.temperature <= 0.0) {
        // greedy: first index of the maximum (AggregationFeatures.java:111-121)
        float bv = -FLT_MAX;
        int bi = INT_MAX;
        for (int i = tid; i < V; i += kSampThreads)
            if (lg[i] > bv) { bv = lg[i]; bi = i; }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        __shared__ float wv[kSampWarps];
        __shared__ int wi[kSampWarps];
        if ((tid & 31) == 0) { wv[tid >> 5] = bv; wi[tid >> 5] = bi; }
        __syncthreads();
        if (tid == 0) {
            bv = wv[0]; bi = wi[0];
            for (int w = 1; w < kSampWarps; w++)
                if (wv[w] > bv || (wv[w] == bv && wi[w] < bi)) { bv = wv[w]; bi = wi[w]; }
            s_pick = bi;
        }
        __syncthreads();
        token = s_pick;
    } else {
        // ---- softmax of logits / temperature (double) ----
        const double T = a.temperature;
        double m = -DBL_MAX;
        for (int i = tid; i < V; i += kSampThreads) m = fmax(m, (double)lg[i] / T);
        m = block_max_d(m, red);
        double s = 0.0;
        for (int i = tid; i < V; i += kSampThreads) {
            const double e = exp((double)lg[i] / T - m);
            q[i] = e;
            s += e;
        }
        s = block_sum_d(s, red);
        for (int i = tid; i < V; i += kSampThreads) q[i] = q[i] / s;
        if (a.mode == 0) {
            // AutoregressiveModel.of: sampleToken(probabilities, vocab, 1.0, 1.0, random) softmaxes again
            double m2 = -DBL_MAX;
            for (int i = tid; i < V; i += kSampThreads) m2 = fmax(m2, q[i]);
            m2 = block_max_d(m2, red);
            double s2 = 0.0;
            for (int i = tid; i < V; i += kSampThreads) {
                const double e = exp(q[i] - m2);
                q[i] = e;
                s2 += e;
            }
            s2 = block_sum_d(s2, red);
            for (int i = tid; i < V; i += kSampThreads) q[i] = q[i] / s2;
        }
        __syncthreads();
        // ---- nucleus filter (mode 1, top_p < 1): radix-select the cutoff probability ----
        double top_sum = 1.0;
        unsigned long long cut = 0;  // elements with bit pattern > cut are kept; == cut kept up to `ties`
        long long ties = -1;         // -1: no filtering
        if (a.mode == 1 && a.top_p < 1.0) {
            // probability mass in 2^-60 fixed point: integer atomics add in any order to the same total, so
            // the cutoff does not depend on the order in which threads arrive (the sum's rounding, at most
            // V x 2^-61 ~ 1e-13, is below any gap the comparison with top_p could resolve in double)
            constexpr double kFix = 1152921504606846976.0;  // 2^60
            unsigned long long *hist_u = reinterpret_cast<unsigned long long *>(hist_m);
            const unsigned long long top_u = __double2ull_rn(a.top_p * kFix);
            unsigned long long prefix = 0;
            unsigned long long above_u = 0;  // mass of the elements whose pattern is above the current prefix range
            const int widths[6] = {11, 11, 11, 11, 10, 10};
            int shift = 64;
            for (int pass = 0; pass < 6; pass++) {
                const int w = widths[pass];
                shift -= w;
                const int nb = 1 << w;
                for (int b = tid; b < nb; b += kSampThreads) hist_u[b] = 0ull;
                __syncthreads();
                const unsigned long long hmask = shift + w >= 64 ? 0ULL : (~0ULL << (shift + w));
                for (int i = tid; i < V; i += kSampThreads) {
                    const double v = q[i];
                    const unsigned long long bits = (unsigned long long)__double_as_longlong(v);
                    if ((bits & hmask) == prefix) atomicAdd(&hist_u[(bits >> shift) & (nb - 1)], __double2ull_rn(v * kFix));
                }
                __syncthreads();
                if (tid == 0) {
                    unsigned long long cum = above_u;
                    int sel = 0;
                    for (int b = nb - 1; b >= 0; b--) {
                        if (cum + hist_u[b] >= top_u) { sel = b; break; }
                        cum += hist_u[b];
                    }
                    s_cum = cum;
                    s_sel = prefix | ((unsigned long long)sel << shift);
                }
                __syncthreads();
                above_u = s_cum;
                prefix = s_sel;
                __syncthreads();
            }
            const double above = (double)above_u / kFix;
            cut = prefix;
            // ties at the cutoff value are taken in index order until the cumulative mass reaches top_p
            const double vc = __longlong_as_double((long long)cut);
            const double need = a.top_p - above;
            long long k = vc > 0.0 ? (long long)ceil(need / vc) : 0;
            if (k < 1) k = 1;
            ties = k;
            top_sum = above + (double)k * vc;
        }
        // ---- categorical draw in index order ----
        if (tid == 0) {
            double r;
            if (a.r) r = a.r[row];
            else {
                unsigned long long st = a.rng[row];
                r = jr_next_double(st);
                a.rng[row] = st;
            }
            s_r = r;
        }
        __syncthreads();
        const double r = s_r;
        const int chunk = (V + kSampThreads - 1) / kSampThreads;
        const int c0 = tid * chunk, c1 = min(V, c0 + chunk);
        // per-thread mass of its index range; ties at the cutoff counted in index order need a prefix
        // count of equal elements first
        long long eq_before = 0;
        if (ties >= 0) {
            long long eq = 0;
            for (int i = c0; i < c1; i++) eq += (unsigned long long)__double_as_longlong(q[i]) == cut;
            // exclusive scan of eq over threads
            __shared__ long long scan_ll[kSampThreads];
            scan_ll[tid] = eq;
            __syncthreads();
            if (tid == 0) {
                long long acc = 0;
                for (int t = 0; t < kSampThreads; t++) { const long long e = scan_ll[t]; scan_ll[t] = acc; acc += e; }
            }
            __syncthreads();
            eq_before = scan_ll[tid];
        }
        auto weight = [&](int i, long long &eq_seen) -> double {
            const double v = q[i];
            if (ties < 0) return v;
            const unsigned long long bits = (unsigned long long)__double_as_longlong(v);
            if (bits > cut) return v / top_sum;
            if (bits == cut) return (eq_seen++ < ties) ? v / top_sum : 0.0;
            return 0.0;
        };
        double part = 0.0;
        {
            long long eqs = eq_before;
            for (int i = c0; i < c1; i++) part += weight(i, eqs);
        }
        __shared__ double scan_d[kSampThreads];
        scan_d[tid] = part;
        __syncthreads();
        if (tid == 0) {  // exclusive scan of the per-thread masses; the thread whose range holds r
            double acc = 0.0;
            int owner = -1;
            for (int t = 0; t < kSampThreads; t++) {
                const double e = scan_d[t];
                scan_d[t] = acc;
                if (owner < 0 && r < acc + e) owner = t;
                acc += e;
            }
            s_pick = owner;
            s_sel = (unsigned long long)(V - 1);  // r beyond the total (rounding): the last index
        }
        __syncthreads();
        if (tid == s_pick) {
            double cum = scan_d[tid];
            long long eqs = eq_before;
            int found = c1 - 1;
            for (int i = c0; i < c1; i++) {
                cum += weight(i, eqs);
                if (r < cum) { found = i; break; }
            }
            s_sel = (unsigned long long)found;
        }
        __syncthreads();
        token = (int)s_sel;
    }
    if (tid == 0) {
        if (a.out) a.out[row] = token;
        if (a.hist) a.hist[(size_t)row * a.hist_ld + a.positions[row] + 1] = token;
        if (a.advance) {
            a.next_tokens[row] = token;
            a.positions[row] += 1;
        }
    }
}

}  // namespace

cudaError_t sample_rows_launch(const SampleArgs &a, int rows, cudaStream_t st) {
    if (rows < 1 || a.V < 1) return cudaErrorInvalidValue;
    qw_sample_rows_kernel<<<rows, kSampThreads, 0, st>>>(a);
    return cudaGetLastError();
}

// scrambled java.util.Random state for new Random(seed)
unsigned long long java_random_state(long long seed) {
    return ((unsigned long long)seed ^ 0x5DEECE66DULL) & ((1ULL << 48) - 1);
}

}  // namespace qw

// qw_gemv.cu -- batch <= 4 decode projections as HBM-streaming GEMV kernels.
//
// One kernel per projection of the decode step, with the neighbouring element-wise work
// fused in:
//   prologue  embedding-row gather (Qwen3.java:414 / AutoregressiveModel.java:430), optional
//             all-reduced partial add, rmsnorm (NormalizationLayerFeatures.java:587-603) into
//             shared memory, residual-stream materialisation by CTA 0;
//   main      y = W x for W (N, K) row-major (LayerFeatures.dense, LayerFeatures.java:785-830),
//             each warp owns two output rows, every lane streams 16-byte chunks of both rows
//             with no L1 allocation (weights are read exactly once per step);
//   epilogue  STORE (+bias), RESID (x_out = x_in + y; SequentialBlock.accum,
//             SequentialBlock.java:413-429), SWIGLU (up * silu(gate), FeedForwardFeatures.java:147-156,
//             gate/up rows interleaved in blocks of 16), ARGMAX (logits + first-index-of-max,
//             AggregationFeatures.java:111-121, reduced by the last CTA to finish).
// The roofline is HBM bandwidth: algorithmic bytes = N*K*sizeof(WT) per launch.
#include "qw_internal.cuh"
#include <float.h>
#include <limits.h>
#include <map>
#include <mutex>

namespace qw {

template <typename WT> struct WUnpack;
template <> struct WUnpack<__nv_bfloat16> {
    static constexpr int V = 8;
    static __device__ __forceinline__ void run(const uint4 &w, float *f) {
        f[0] = bf16lo(w.x); f[1] = bf16hi(w.x); f[2] = bf16lo(w.y); f[3] = bf16hi(w.y);
        f[4] = bf16lo(w.z); f[5] = bf16hi(w.z); f[6] = bf16lo(w.w); f[7] = bf16hi(w.w);
    }
};
template <> struct WUnpack<float> {
    static constexpr int V = 4;
    static __device__ __forceinline__ void run(const uint4 &w, float *f) {
        f[0] = __uint_as_float(w.x); f[1] = __uint_as_float(w.y);
        f[2] = __uint_as_float(w.z); f[3] = __uint_as_float(w.w);
    }
};

template <int V>
__device__ __forceinline__ float dotv(const float *f, const float *x) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < V; i += 4) {
        float4 xv = *reinterpret_cast<const float4 *>(x + i);
        s = fmaf(f[i + 0], xv.x, s);
        s = fmaf(f[i + 1], xv.y, s);
        s = fmaf(f[i + 2], xv.z, s);
        s = fmaf(f[i + 3], xv.w, s);
    }
    return s;
}

template <typename WT>
__device__ __forceinline__ float4 load4(const WT *p);
template <> __device__ __forceinline__ float4 load4<float>(const float *p) {
    return *reinterpret_cast<const float4 *>(p);
}
template <> __device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16 *p) {
    uint2 u = *reinterpret_cast<const uint2 *>(p);
    return make_float4(bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y));
}

constexpr int kGemvThreads = 256;
constexpr int kGemvUnroll = 4;

template <typename WT, int EPI, int NB>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(16) float xs[];  // [NB][K]
    __shared__ float red[NB][kGemvThreads / 32];
    __shared__ int redi[NB][kGemvThreads / 32];
    __shared__ int s_is_last;
    const int K = a.K;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = kGemvThreads / 32;

    // ---------------- prologue: activation row(s) -> shared memory ----------------
    float ss[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) {
        ss[b] = 0.f;
        const WT *erow = a.embed ? reinterpret_cast<const WT *>(a.embed) + (size_t)a.tokens[b] * K : nullptr;
        for (int k = tid * 4; k < K; k += kGemvThreads * 4) {
            float4 v = erow ? load4<WT>(erow + k) : *reinterpret_cast<const float4 *>(a.xin + (size_t)b * a.ld_in + k);
            if (a.part) {
                float4 p = *reinterpret_cast<const float4 *>(a.part + (size_t)b * a.ld_part + k);
                v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
            }
            if (a.xsave && blockIdx.x == 0) *reinterpret_cast<float4 *>(a.xsave + (size_t)b * a.ld_xsave + k) = v;
            *reinterpret_cast<float4 *>(xs + b * K + k) = v;
            ss[b] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
    }
    if (a.norm_w) {
#pragma unroll
        for (int b = 0; b < NB; b++) {
            float s = warp_sum(ss[b]);
            if (lane == 0) red[b][warp] = s;
        }
        __syncthreads();
#pragma unroll
        for (int b = 0; b < NB; b++) {
            float s = 0.f;
#pragma unroll
            for (int w = 0; w < NW; w++) s += red[b][w];
            ss[b] = 1.0f / sqrtf(s / (float)K + a.eps);
        }
#pragma unroll
        for (int b = 0; b < NB; b++)
            for (int k = tid * 4; k < K; k += kGemvThreads * 4) {
                float4 v = *reinterpret_cast<float4 *>(xs + b * K + k);
                float4 w = *reinterpret_cast<const float4 *>(a.norm_w + k);
                v.x = w.x * v.x * ss[b]; v.y = w.y * v.y * ss[b];
                v.z = w.z * v.z * ss[b]; v.w = w.w * v.w * ss[b];
                *reinterpret_cast<float4 *>(xs + b * K + k) = v;
            }
    }
    __syncthreads();

    // ---------------- main: two rows per warp, contiguous task range per CTA ----------------
    constexpr int V = WUnpack<WT>::V;
    const int nch = K / V;
    const int ntask = (EPI == EPI_SWIGLU) ? a.N / 2 : (a.N + 1) / 2;
    const int t_begin = (int)(((long long)ntask * blockIdx.x) / gridDim.x);
    const int t_end = (int)(((long long)ntask * (blockIdx.x + 1)) / gridDim.x);
    const size_t row_bytes = (size_t)K * sizeof(WT);
    const char *Wb = reinterpret_cast<const char *>(a.W);

    float bestv[NB];
    int besti[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) { bestv[b] = -FLT_MAX; besti[b] = INT_MAX; }

    for (int task = t_begin + warp; task < t_end; task += NW) {
        int r0, r1;
        bool v1;
        if (EPI == EPI_SWIGLU) {
            r0 = (task / kGuBlock) * (2 * kGuBlock) + (task % kGuBlock);
            r1 = r0 + kGuBlock;
            v1 = true;
        } else {
            r0 = 2 * task;
            v1 = (r0 + 1) < a.N;
            r1 = v1 ? r0 + 1 : r0;
        }
        const uint4 *w0 = reinterpret_cast<const uint4 *>(Wb + (size_t)r0 * row_bytes);
        const uint4 *w1 = reinterpret_cast<const uint4 *>(Wb + (size_t)r1 * row_bytes);
        float acc0[NB], acc1[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) { acc0[b] = 0.f; acc1[b] = 0.f; }

        for (int c0 = lane; c0 < nch; c0 += 32 * kGemvUnroll) {
            uint4 u0[kGemvUnroll], u1[kGemvUnroll];
#pragma unroll
            for (int i = 0; i < kGemvUnroll; i++) {
                int c = c0 + 32 * i;
                if (c < nch) { u0[i] = ld_stream(w0 + c); u1[i] = ld_stream(w1 + c); }
            }
#pragma unroll
            for (int i = 0; i < kGemvUnroll; i++) {
                int c = c0 + 32 * i;
                if (c < nch) {
                    float f0[V], f1[V];
                    WUnpack<WT>::run(u0[i], f0);
                    WUnpack<WT>::run(u1[i], f1);
#pragma unroll
                    for (int b = 0; b < NB; b++) {
                        const float *xv = xs + b * K + c * V;
                        acc0[b] += dotv<V>(f0, xv);
                        acc1[b] += dotv<V>(f1, xv);
                    }
                }
            }
        }
#pragma unroll
        for (int b = 0; b < NB; b++) { acc0[b] = warp_sum(acc0[b]); acc1[b] = warp_sum(acc1[b]); }

        if (lane == 0) {
#pragma unroll
            for (int b = 0; b < NB; b++) {
                if (EPI == EPI_STORE) {
                    float* o = a.out + (size_t)b * a.ld_out;
                    o[r0] = acc0[b] + (a.bias ? a.bias[r0] : 0.f);
                    if (v1) o[r1] = acc1[b] + (a.bias ? a.bias[r1] : 0.f);
                } else if (EPI == EPI_RESID) {
                    float* o = a.out + (size_t)b * a.ld_out;
                    const float *rs = a.resid ? a.resid + (size_t)b * a.ld_resid : nullptr;
                    o[r0] = (rs ? rs[r0] : 0.f) + acc0[b];
                    if (v1) o[r1] = (rs ? rs[r1] : 0.f) + acc1[b];
                } else if (EPI == EPI_SWIGLU) {
                    float g = acc0[b], u = acc1[b];
                    float sg = 1.0f / (1.0f + expf(-g));
                    a.out[(size_t)b * a.ld_out + task] = u * (g * sg);
                } else {  // EPI_ARGMAX
                    if (a.out) {
                        float* o = a.out + (size_t)b * a.ld_out;
                        o[r0] = acc0[b];
                        if (v1) o[r1] = acc1[b];
                    }
                    if (acc0[b] > bestv[b]) { bestv[b] = acc0[b]; besti[b] = r0; }
                    if (v1 && acc1[b] > bestv[b]) { bestv[b] = acc1[b]; besti[b] = r1; }
                }
            }
        }
    }

    if (EPI == EPI_ARGMAX) {
        // CTA reduction (ties -> smaller index), then the last CTA reduces over the grid.
        if (lane == 0) {
#pragma unroll
            for (int b = 0; b < NB; b++) { red[b][warp] = bestv[b]; redi[b][warp] = besti[b]; }
        }
        __syncthreads();
        if (tid < NB) {
            float bv = -FLT_MAX;
            int bi = INT_MAX;
            for (int w = 0; w < NW; w++) {
                float v = red[tid][w];
                int i = redi[tid][w];
                if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
            }
            a.part_val[blockIdx.x * NB + tid] = bv;
            a.part_idx[blockIdx.x * NB + tid] = bi;
            __threadfence();
        }
        __syncthreads();
        if (tid == 0) {
            unsigned t = atomicAdd(a.counter, 1u);
            s_is_last = (t == gridDim.x - 1);
        }
        __syncthreads();
        if (s_is_last) {
            __threadfence();
            for (int b = warp; b < NB; b += NW) {
                float bv = -FLT_MAX;
                int bi = INT_MAX;
                for (int c = lane; c < (int)gridDim.x; c += 32) {
                    float v = __ldcg(a.part_val + c * NB + b);
                    int i = __ldcg(a.part_idx + c * NB + b);
                    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
                }
                if (lane == 0) {
                    int g = bi + a.idx_offset;
                    if (a.argmax_out) a.argmax_out[b] = g;
                    if (a.argmax_val) a.argmax_val[b] = bv;
                    if (a.hist) a.hist[(size_t)b * a.hist_ld + a.positions[b] + 1] = g;
                    if (a.advance) {
                        a.next_tokens[b] = g;
                        a.positions[b] += 1;
                    }
                }
            }
            if (tid == 0) *a.counter = 0u;
        }
    }
}

// ---------------------------------------------------------------------------------------------
// launcher
// ---------------------------------------------------------------------------------------------
// Opt the kernel in to `smem` bytes of dynamic shared memory and return its blocks per SM;
// cached per (kernel, smem) so the attribute calls happen once, outside of stream capture.
static int prepare_cached(const void *fn, size_t smem, cudaError_t *err) {
    static std::mutex mu;
    static std::map<std::pair<const void *, size_t>, int> cache;
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find({fn, smem});
    if (it != cache.end()) return it->second;
    *err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (*err != cudaSuccess) return 0;
    int occ = 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, kGemvThreads, smem) != cudaSuccess || occ < 1) occ = 1;
    cache[{fn, smem}] = occ;
    return occ;
}

template <typename WT, int EPI, int NB>
static cudaError_t launch_t(const GemvArgs &a, int num_sms, cudaStream_t st) {
    size_t smem = (size_t)NB * a.K * sizeof(float);
    auto kfn = gemv_kernel<WT, EPI, NB>;
    cudaError_t e = cudaSuccess;
    int occ = prepare_cached((const void *)kfn, smem, &e);
    if (e != cudaSuccess) return e;
    int ntask = (EPI == EPI_SWIGLU) ? a.N / 2 : (a.N + 1) / 2;
    int want = (ntask + (kGemvThreads / 32) - 1) / (kGemvThreads / 32);
    int cap = num_sms * occ;
    int grid = want < cap ? (want > 0 ? want : 1) : cap;
    kfn<<<grid, kGemvThreads, smem, st>>>(a);
    return cudaGetLastError();
}

template <typename WT, int EPI>
static cudaError_t launch_b(const GemvArgs &a, int num_sms, cudaStream_t st) {
    switch (a.B) {
        case 1: return launch_t<WT, EPI, 1>(a, num_sms, st);
        case 2: return launch_t<WT, EPI, 2>(a, num_sms, st);
        case 3: return launch_t<WT, EPI, 3>(a, num_sms, st);
        case 4: return launch_t<WT, EPI, 4>(a, num_sms, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t gemv_launch(const GemvArgs &a, int epi, bool bf16, int num_sms, cudaStream_t st) {
    if (a.B < 1 || a.B > kGemvMaxB || (a.K % 8) != 0) return cudaErrorInvalidValue;
    if (bf16) {
        switch (epi) {
            case EPI_STORE: return launch_b<__nv_bfloat16, EPI_STORE>(a, num_sms, st);
            case EPI_RESID: return launch_b<__nv_bfloat16, EPI_RESID>(a, num_sms, st);
            case EPI_SWIGLU: return launch_b<__nv_bfloat16, EPI_SWIGLU>(a, num_sms, st);
            case EPI_ARGMAX: return launch_b<__nv_bfloat16, EPI_ARGMAX>(a, num_sms, st);
        }
    } else {
        switch (epi) {
            case EPI_STORE: return launch_b<float, EPI_STORE>(a, num_sms, st);
            case EPI_RESID: return launch_b<float, EPI_RESID>(a, num_sms, st);
            case EPI_SWIGLU: return launch_b<float, EPI_SWIGLU>(a, num_sms, st);
            case EPI_ARGMAX: return launch_b<float, EPI_ARGMAX>(a, num_sms, st);
        }
    }
    return cudaErrorInvalidValue;
}

}  // namespace qw

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
#include "qw_ops.h"
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
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kGemvRows = 4;    // rows per CTA tile (SWIGLU: 2 gate + the 2 matching up rows)
constexpr int kGemvUnroll = 2;  // 16-byte chunks per lane per row per k-step (8 loads in flight per lane)

template <int EPI>
__device__ __forceinline__ int tile_row(int tile, int r) {
    if (EPI == EPI_SWIGLU) {
        int pair = tile * (kGemvRows / 2) + (r % (kGemvRows / 2));
        int gate = (pair / kGuBlock) * (2 * kGuBlock) + (pair % kGuBlock);
        return r < kGemvRows / 2 ? gate : gate + kGuBlock;
    }
    return tile * kGemvRows + r;
}

// Issue the weight loads of one pipeline stage (one k-step of one row tile) into registers.
template <typename WT, int EPI>
__device__ __forceinline__ void gemv_issue(uint4 (&u)[kGemvRows][kGemvUnroll], const char *Wb, size_t row_bytes,
                                           int N, int nch, int tile, int kstep, int warp, int lane) {
    constexpr int NW = kGemvWarps, U = kGemvUnroll, STEP = NW * 32 * U;
    const int c0 = kstep * STEP + warp * 32 + lane;
#pragma unroll
    for (int r = 0; r < kGemvRows; r++) {
        const int row = tile_row<EPI>(tile, r);
        const uint4 *w = reinterpret_cast<const uint4 *>(Wb + (size_t)(row < N ? row : 0) * row_bytes);
#pragma unroll
        for (int i = 0; i < U; i++) {
            const int c = c0 + i * NW * 32;
            u[r][i] = (c < nch && row < N) ? ld_stream(w + c) : make_uint4(0, 0, 0, 0);
        }
    }
}

// One CTA streams a contiguous range of row tiles; the 8 warps split K of every tile
// (each warp reads 512 contiguous bytes per row per load), so all warps and all CTAs
// carry the same number of bytes.  Loads run one stage ahead of the FMAs (register double
// buffer), the first stage is issued before the programmatic-launch wait so it overlaps the
// previous kernel's tail, and partial sums meet in shared memory once per tile.
template <typename WT, int EPI, int NB>
__global__ void __launch_bounds__(kGemvThreads) qw_gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(16) float xs[];  // [NB][K]
    __shared__ float red[2][kGemvWarps][kGemvRows * NB];
    __shared__ float am_v[kGemvRows * NB];
    __shared__ int am_i[kGemvRows * NB];
    __shared__ int s_is_last;
    const int K = a.K;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = kGemvWarps;
    constexpr int R = kGemvRows;
    constexpr int U = kGemvUnroll;
    constexpr int V = WUnpack<WT>::V;
    constexpr int STEP = NW * 32 * U;  // 16-byte chunks per k-step of the whole CTA

    const int nch = K / V;
    const int N = a.N;
    const int ntiles = (EPI == EPI_SWIGLU) ? (N / 2) / (R / 2) : (N + R - 1) / R;
    const int t_begin = (int)(((long long)ntiles * blockIdx.x) / gridDim.x);
    const int t_end = (int)(((long long)ntiles * (blockIdx.x + 1)) / gridDim.x);
    const size_t row_bytes = (size_t)K * sizeof(WT);
    const char *Wb = reinterpret_cast<const char *>(a.W);
    const int ksteps = (nch + STEP - 1) / STEP;
    const int nstage = (t_end - t_begin) * ksteps;

    // weights do not depend on the previous kernel: start streaming them before the wait
    uint4 ucur[R][U], unext[R][U];
    if (nstage > 0) gemv_issue<WT, EPI>(ucur, Wb, row_bytes, N, nch, t_begin, 0, warp, lane);
    griddep_wait();
    griddep_launch_dependents();

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
            if (lane == 0) red[0][warp][b] = s;
        }
        __syncthreads();
#pragma unroll
        for (int b = 0; b < NB; b++) {
            float s = 0.f;
#pragma unroll
            for (int w = 0; w < NW; w++) s += red[0][w][b];
            ss[b] = 1.0f / sqrtf(s / (float)K + a.eps);
        }
        __syncthreads();
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

    // ---------------- main: pipelined stages ----------------
    float bestv = -FLT_MAX;  // ARGMAX: per epilogue thread (r, b)
    int besti = INT_MAX;
    float acc[R][NB];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int b = 0; b < NB; b++) acc[r][b] = 0.f;
    int buf = 0;
    for (int st = 0; st < nstage; st++) {
        const int tile = t_begin + st / ksteps, kstep = st % ksteps;
        if (st + 1 < nstage)
            gemv_issue<WT, EPI>(unext, Wb, row_bytes, N, nch, t_begin + (st + 1) / ksteps, (st + 1) % ksteps, warp,
                                lane);
        const int c0 = kstep * STEP + warp * 32 + lane;
#pragma unroll
        for (int i = 0; i < U; i++) {
            const int c = c0 + i * NW * 32;
            if (c < nch) {
#pragma unroll
                for (int b = 0; b < NB; b++) {
                    float xv[V];
#pragma unroll
                    for (int j = 0; j < V; j += 4) {
                        float4 t4 = *reinterpret_cast<const float4 *>(xs + b * K + c * V + j);
                        xv[j] = t4.x; xv[j + 1] = t4.y; xv[j + 2] = t4.z; xv[j + 3] = t4.w;
                    }
#pragma unroll
                    for (int r = 0; r < R; r++) {
                        float f[V];
                        WUnpack<WT>::run(ucur[r][i], f);
                        float sacc = acc[r][b];
#pragma unroll
                        for (int j = 0; j < V; j++) sacc = fmaf(f[j], xv[j], sacc);
                        acc[r][b] = sacc;
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
            for (int i = 0; i < U; i++) ucur[r][i] = unext[r][i];
        if (kstep != ksteps - 1) continue;

        // ---- tile complete: reduce over warps, epilogue ----
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
            for (int b = 0; b < NB; b++) {
                float v = warp_sum(acc[r][b]);
                acc[r][b] = 0.f;
                if (lane == 0) red[buf][warp][r * NB + b] = v;
            }
        __syncthreads();
        if (tid < R * NB) {
            const int r = tid / NB, b = tid % NB;
            float y = 0.f;
#pragma unroll
            for (int w = 0; w < NW; w++) y += red[buf][w][tid];
            const int row = tile_row<EPI>(tile, r);
            if (EPI == EPI_STORE) {
                if (row < N) a.out[(size_t)b * a.ld_out + row] = y + (a.bias ? a.bias[row] : 0.f);
            } else if (EPI == EPI_RESID) {
                if (row < N)
                    a.out[(size_t)b * a.ld_out + row] = (a.resid ? a.resid[(size_t)b * a.ld_resid + row] : 0.f) + y;
            } else if (EPI == EPI_SWIGLU) {
                if (r < R / 2) {
                    float g = y;
                    float u = 0.f;
#pragma unroll
                    for (int w = 0; w < NW; w++) u += red[buf][w][(r + R / 2) * NB + b];
                    float sg = 1.0f / (1.0f + expf(-g));
                    int pair = tile * (R / 2) + r;
                    a.out[(size_t)b * a.ld_out + pair] = u * (g * sg);
                }
            } else {  // EPI_ARGMAX: rows increase within a thread, so strict > keeps the first max
                if (row < N) {
                    if (a.out) a.out[(size_t)b * a.ld_out + row] = y;
                    if (y > bestv) { bestv = y; besti = row; }
                }
            }
        }
        buf ^= 1;
    }

    if (EPI == EPI_ARGMAX) {
        if (tid < R * NB) { am_v[tid] = bestv; am_i[tid] = besti; }
        __syncthreads();
        if (tid < NB) {
            float bv = -FLT_MAX;
            int bi = INT_MAX;
            for (int r = 0; r < R; r++) {
                float v = am_v[r * NB + tid];
                int i = am_i[r * NB + tid];
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
    // one opt-in to the largest size per kernel: a smaller later setting would invalidate
    // launches of larger, already-cached sizes
    static std::map<const void *, bool> opted;
    if (!opted[fn]) {
        int dev = 0, optin = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        int stat_smem = 4096;  // static shared memory margin
        *err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - stat_smem);
        if (*err != cudaSuccess) return 0;
        opted[fn] = true;
    }
    int occ = 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, kGemvThreads, smem) != cudaSuccess || occ < 1) occ = 1;
    // the argmax epilogue's cross-CTA scratch (qw_ops.cu, qw_noalloc.cu) is sized for this many CTAs per SM
    if (occ > kGemvMaxCtasPerSm) occ = kGemvMaxCtasPerSm;
    cache[{fn, smem}] = occ;
    return occ;
}

template <typename WT, int EPI, int NB>
static cudaError_t launch_t(const GemvArgs &a, int num_sms, cudaStream_t st) {
    size_t smem = (size_t)NB * a.K * sizeof(float);
    auto kfn = qw_gemv_kernel<WT, EPI, NB>;
    cudaError_t e = cudaSuccess;
    int occ = prepare_cached((const void *)kfn, smem, &e);
    if (e != cudaSuccess) return e;
    // persistent grid: every SM holds `occ` CTAs for the whole launch
    int ntiles = (EPI == EPI_SWIGLU) ? (a.N / 2) / (kGemvRows / 2) : (a.N + kGemvRows - 1) / kGemvRows;
    int cap = num_sms * occ;
    int grid = ntiles < cap ? (ntiles > 0 ? ntiles : 1) : cap;
    return launch_pdl(kfn, dim3(grid), dim3(kGemvThreads), smem, st, a);
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

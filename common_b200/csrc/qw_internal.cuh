// qw_internal.cuh -- shared device helpers and kernel argument blocks for libqwen3_b200.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string.h>
#include <utility>

#define QW_WARP 32

namespace qw {

constexpr int kNumSMsB200 = 148;

// ---------------------------------------------------------------------------------------------
// element helpers
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float bf16lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }

// round-to-nearest-even fp32 -> bf16 bits (NaN kept quiet)
__host__ __device__ __forceinline__ uint16_t f2bf_bits(float f) {
#ifdef __CUDA_ARCH__
    uint32_t u = __float_as_uint(f);
#else
    uint32_t u;
    memcpy(&u, &f, 4);
#endif
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
__device__ __forceinline__ float bf_round(float f) { return __uint_as_float((uint32_t)f2bf_bits(f) << 16); }

template <typename T> struct Elt;
template <> struct Elt<float> {
    static __device__ __forceinline__ float load(const float *p) { return *p; }
    static __device__ __forceinline__ void store(float *p, float v) { *p = v; }
    static __device__ __forceinline__ float round(float v) { return v; }
};
template <> struct Elt<__nv_bfloat16> {
    static __device__ __forceinline__ float load(const __nv_bfloat16 *p) {
        return __uint_as_float((uint32_t)(*(const uint16_t *)p) << 16);
    }
    static __device__ __forceinline__ void store(__nv_bfloat16 *p, float v) { *(uint16_t *)p = f2bf_bits(v); }
    static __device__ __forceinline__ float round(float v) { return bf_round(v); }
};

// streaming 16-byte load: read-only path, no L1 allocation (weights are touched once per step)
__device__ __forceinline__ uint4 ld_stream(const void *p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    return r;
}

// programmatic dependent launch: let the next kernel in the stream start its independent
// prologue, and wait for the previous kernel's results before touching them
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// counter-based synthetic generator; bit-identical to oref_synth_value in the oracle:
// splitmix64 of (seed, tensor id, index) -> Irwin-Hall sum of four 16-bit uniforms * scale.
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__host__ __device__ __forceinline__ float synth_value(uint64_t seed, uint32_t tensor_id, uint64_t idx, float scale) {
    uint64_t h = splitmix64(seed ^ ((uint64_t)tensor_id << 40) ^ splitmix64(idx));
    int s = (int)(h & 0xFFFF) + (int)((h >> 16) & 0xFFFF) + (int)((h >> 32) & 0xFFFF) + (int)(h >> 48) - 2 * 65535;
    return (float)s * scale;
}

// ---------------------------------------------------------------------------------------------
// GEMV (batch <= kGemvMaxB decode) argument block
// ---------------------------------------------------------------------------------------------
constexpr int kGemvMaxB = 4;
constexpr int kGuBlock = 16;  // gate/up rows interleaved in blocks of 16 (gate rows, then up rows)

enum GemvEpi { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3 };

struct GemvArgs {
    const void *W;  // (N, K) row-major, storage type WT
    int N, K;
    int B;
    // prologue: x_b = src_b (+ part_b); optionally rmsnorm(x_b) * norm_w
    const float *xin;  // (B, ld_in) fp32 (ignored when embed != nullptr)
    int ld_in;
    const float *part;  // optional all-reduced partial added to xin
    int ld_part;
    const void *embed;  // optional (vocab, K) table in WT: x_b = embed[tokens[b]]
    const int *tokens;
    const float *norm_w;  // optional rmsnorm weight (K)
    float eps;
    float *xsave;  // optional: CTA 0 writes the un-normalised x_b here (residual stream)
    int ld_xsave;
    // epilogue
    float *out;  // STORE/RESID: (B, ld_out); SWIGLU: (B, ld_out) with N/2 columns; ARGMAX: logits (nullable)
    int ld_out;
    const float *resid;  // RESID: out = resid + y (nullable -> out = y)
    int ld_resid;
    const float *bias;  // STORE: optional bias (N)
    // ARGMAX
    float *part_val;  // (gridDim.x, B)
    int *part_idx;
    unsigned *counter;  // 1 element, zero on entry, reset by the last CTA
    int idx_offset;     // global index of row 0 (vocab shard start)
    int *argmax_out;    // (B) final winner (global index); nullable when tp > 1
    float *argmax_val;  // (B) winning value (for cross-rank reduction); nullable
    int *next_tokens;   // advance: tokens[b] = winner
    int *positions;     // advance: positions[b] += 1
    int advance;
    int *hist;          // optional: hist[b * hist_ld + positions[b] + 1] = winner (generation record)
    int hist_ld;
};

// ---------------------------------------------------------------------------------------------
// decode attention argument block
// ---------------------------------------------------------------------------------------------
struct AttnArgs {
    const float *qkv;  // (B, ld_qkv): q (H_local*d) | k (Hkv_local*d) | v (Hkv_local*d)
    int ld_qkv;
    const float *qn, *kn;  // q_norm / k_norm weights of this rank's heads (nullable when mode 0)
    int qk_mode;           // 0 none, 1 whole vector, 2 per head
    const float *qk_ss;    // optional (B, 2) global sums of squares (vector mode, tp > 1)
    int q_total, kv_total; // global q / kv widths for the vector norm
    const float2 *freq;    // (seq_len, d/2) cos, sin
    void *kcache, *vcache; // this layer: [page][Hkv_local][page_size][d]
    const int *page_table; // [slot][max_pages]
    int max_pages;
    const int *slots;      // (B) nullable -> b
    const int *positions;  // (B)
    int H, Hkv, d, page_size, log2_page;
    int nsplit;
    float scale;           // 1/sqrt(d)
    float *part_o;         // (B, H, nsplit, d)
    float *part_ml;        // (B, H, nsplit, 2)
    unsigned *counters;    // (B, Hkv), zero on entry
    float *out;            // (B, ld_out) attention output, head-major
    int ld_out;
    __nv_bfloat16 *out_bf16;  // optional: bf16 output (B, ld_out) instead of `out`
};

}  // namespace qw

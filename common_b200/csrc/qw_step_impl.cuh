// qw_step_impl.cuh -- the whole batch-1 decode step as one persistent kernel (included by qw_step.cu,
// which instantiates it for tp = 1, and qw_step_tp.cu, which instantiates the tensor-parallel variants).
//
// Batch-1 decode streams every weight byte once per token; its speed is set by how close the
// weight stream stays to HBM bandwidth.  Launching one kernel per projection loses that at every
// boundary (ramp-up, tail, prologue), so here one CTA per SM runs the full step
// (Qwen3.java:334-415: L x [rmsnorm, QKV, QK-norm, RoPE, KV write, attention, O + residual,
// rmsnorm, gate/up, SwiGLU, down + residual], final rmsnorm, lm_head, greedy argmax):
//
//   warp 8 (producer)   streams this CTA's contiguous share of every weight matrix of the step,
//                       in step order, into a ring of 16 KiB shared-memory slots with
//                       cp.async.bulk (no multicast).  It only waits for free slots, never for
//                       activations, so HBM keeps streaming the next phase's weights while the
//                       consumers sit in a grid barrier or in the attention phase.
//   warps 0-7           consume the slots: 8-element bf16 x fp32 dot products against the phase's
//                       activation vector (fp32, in shared memory), per-row partial sums in
//                       shared memory, the phase epilogue, then a grid barrier.
//
// Phases per layer: QKV (rows split over CTAs) | attention (work items = KV head x context
// split, merged by the last CTA of each KV head) | O + residual | gate/up (raw, SwiGLU is
// applied by the next phase's loader) | down + residual.  Then lm_head with a first-index-of-max
// reduction (AggregationFeatures.java:111-121) merged by the last CTA, which also feeds the
// token back and advances the position (AutoregressiveModel.java:295-308).
//
// Data written by one CTA and read by another after a grid barrier is read with ld.global.cg
// (L2), never through L1.  Every wait (slot barriers, grid barriers) is bounded by time: on
// expiry the kernel records an error, stops, lets its issued copies land and returns.
#pragma once
#include "qw_internal.cuh"
#include "qw_kernels.h"
#include <float.h>
#include <limits.h>
#include <algorithm>

namespace qw {

namespace {

constexpr int kStepConsumerWarps = 8;
constexpr int kStepConsumers = kStepConsumerWarps * 32;
constexpr int kStepThreads = kStepConsumers + 32;
static_assert(kStepThreads == kStepBlockThreads, "block size");
constexpr int kPiece = 32768;  // bytes per ring slot (16384 bf16 weights: R rows x C columns)
constexpr int kRing = 5;
// layout of a rank's exchange buffer (32-bit words): flags, QK-norm sums, argmax, row partials
constexpr int kXFlags = 0;   // [tp] generation flags, written by each peer
constexpr int kXSs = 64;     // [tp][2] 8-byte words: q / k sums of squares of the current layer, one slot per rank
constexpr int kXAm = 96;     // [tp][2] (value, index) of each rank's vocabulary shard
constexpr int kXRows = 128;  // [2][tp][D] 8-byte words: O partials, then down partials
constexpr int kStepTPW = 4;  // attention: keys per warp per tile (small: this code runs once per layer, cold in the instruction cache)

__device__ __forceinline__ uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
// cycle counter of this SM: cheap to read in a spin loop (the bounds below are in cycles)
__device__ __forceinline__ uint64_t now_ns() { return (uint64_t)clock64(); }
// wall-clock nanoseconds (the profiling trace only)
__device__ __forceinline__ unsigned long long trace_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ bool mb_try(uint32_t addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mb_wait(uint64_t *b, uint32_t parity, volatile int *abort_flag, int *err,
                                        unsigned long long lim) {
    const uint32_t addr = su32(b);
    if (mb_try(addr, parity)) return true;
    const uint64_t t0 = now_ns();
    for (;;) {
        if (mb_try(addr, parity)) return true;
        if (*abort_flag) return false;
        if (now_ns() - t0 > lim) {
            *abort_flag = 1;
            atomicExch(err, 1);
            return false;
        }
    }
}
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kStepConsumers) : "memory"); }

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

template <typename T>
__device__ __forceinline__ T ldcg(const T *p) { return __ldcg(p); }

// context splits of the attention phase: at most one work item per CTA, at least 16 keys per split,
// at most 16 splits
__device__ __forceinline__ int attn_splits(int grid, int Hkv, int n) {
    int ns = min(grid / Hkv, (n + 15) / 16);
    return max(1, min(ns, 16));  // <= 16: the split merge loads every partial in one round
}

__device__ __forceinline__ void split_rows(int N, int c, int n, int &r0, int &r1) {
    r0 = (int)(((long long)N * c) / n);
    r1 = (int)(((long long)N * (c + 1)) / n);
}

struct Ring {
    uint64_t *full, *empty;
    uint8_t *buf;
    int slot;
    uint32_t ph;
    unsigned long long lim;  // wait bound (cycles)
    int row_copies;          // one copy per row even when a slot's rows are contiguous
};

// Column chunk of one ring slot.  A slot holds the same C columns of R = 16384 / C consecutive rows
// (32 KiB of bf16): wide matrices fill a slot with 4 rows of 4096 columns, the narrow K of a
// tensor-parallel shard (K = 512 at tp 8) with 32 rows of 512, so that every slot carries the same bytes
// whatever the shard.  Every activation value read from shared memory serves 4 weight rows.
__host__ __device__ __forceinline__ int chunk_cols(int K) {
    return (K & 4095) == 0 ? 4096 : ((K & 2047) == 0 ? 2048 : ((K & 1023) == 0 ? 1024 : 512));
}
__host__ __device__ __forceinline__ int slot_rows(int C) { return (kPiece / 2) / C; }

// producer: this CTA's rows [r0, r1) of W (N, K), R rows at a time, each group in column chunks.  When a
// chunk spans whole rows (K == C) the group is one contiguous copy.
__device__ __forceinline__ bool produce(Ring &rg, const __nv_bfloat16 *W, int N, int K, volatile int *abort_flag,
                                        int *err, uint32_t &issued, uint32_t &last_ph, uint64_t policy) {
    int r0, r1;
    split_rows(N, blockIdx.x, gridDim.x, r0, r1);
    const int C = chunk_cols(K), R = slot_rows(C);
    for (int ra = r0; ra < r1; ra += R) {
        const int nr = min(R, r1 - ra);
        for (int c0 = 0; c0 < K; c0 += C) {
            if (!mb_wait(&rg.empty[rg.slot], rg.ph ^ 1u, abort_flag, err, rg.lim)) return false;
            const uint32_t fb = su32(&rg.full[rg.slot]);
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(fb), "r"((uint32_t)(nr * C * 2))
                         : "memory");
            const bool whole = C == K && !rg.row_copies;
            const int ncopy = whole ? 1 : nr;
            const uint32_t bytes = (uint32_t)((whole ? nr : 1) * C * 2);
            for (int j = 0; j < ncopy; j++)
                asm volatile(
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
                    "%4;" ::"r"(su32(rg.buf + (size_t)rg.slot * kPiece + (size_t)j * C * 2)),
                    "l"(W + (size_t)(ra + j) * K + c0), "r"(bytes), "r"(fb), "l"(policy)
                    : "memory");
            issued |= 1u << rg.slot;
            last_ph = (last_ph & ~(1u << rg.slot)) | (rg.ph << rg.slot);
            if (++rg.slot == kRing) { rg.slot = 0; rg.ph ^= 1u; }
        }
    }
    return true;
}

__device__ __forceinline__ float dot4(const uint2 w, const float4 x, float acc) {
    acc = fmaf(bf16lo(w.x), x.x, acc);
    acc = fmaf(bf16hi(w.x), x.y, acc);
    acc = fmaf(bf16lo(w.y), x.z, acc);
    return fmaf(bf16hi(w.y), x.w, acc);
}

// Sum four per-lane values over the warp in 6 shuffles: afterwards lane 0 holds the total of v0,
// lane 8 of v1, lane 16 of v2 and lane 24 of v3.
__device__ __forceinline__ float warp_sum4(float v0, float v1, float v2, float v3) {
    const int lane = threadIdx.x & 31;
    const bool lo = lane < 16;
    float x0 = lo ? v0 : v2, x1 = lo ? v1 : v3;
    const float y0 = lo ? v2 : v0, y1 = lo ? v3 : v1;
    x0 += __shfl_xor_sync(0xffffffffu, y0, 16);
    x1 += __shfl_xor_sync(0xffffffffu, y1, 16);
    const bool lo8 = (lane & 8) == 0;
    float z = lo8 ? x0 : x1;
    z += __shfl_xor_sync(0xffffffffu, lo8 ? x1 : x0, 8);
    z += __shfl_xor_sync(0xffffffffu, z, 4);
    z += __shfl_xor_sync(0xffffffffu, z, 2);
    z += __shfl_xor_sync(0xffffffffu, z, 1);
    return z;
}

// consumers: acc[r - r0] = W[r, :] . xs for this CTA's rows.  Every warp takes a 4-row x 512-column block of
// each slot (row block w / (C / 512), column block w % (C / 512)) in 128-column steps, lane l columns
// 4l .. 4l+3 of a step (contiguous 16-byte activation loads, 8-byte weight loads); the partial sums stay in
// registers until the row group is done.  C is a template argument so the slot loop unrolls completely.
template <int C>
__device__ __forceinline__ bool consume_c(Ring &rg, int K, const float *xs, float *acc, int r0, int r1,
                                          volatile int *abort_flag, int *err) {
    constexpr int CB = C / 512;          // column blocks per slot
    constexpr int R = (kPiece / 2) / C;  // rows per slot
    constexpr int STEPS = 4;
    static_assert(R == 4 * (kStepConsumerWarps / CB), "8 warps cover a slot");
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int rb = (warp / CB) * 4, cw = (warp % CB) * 512 + lane * 4;
    for (int ra = r0; ra < r1; ra += R) {
        const int nr = min(R, r1 - ra) - rb;  // rows of this warp's block present in the group (may be <= 0)
        float p[4][STEPS];
#pragma unroll
        for (int r = 0; r < 4; r++)
#pragma unroll
            for (int j = 0; j < STEPS; j++) p[r][j] = 0.f;
        for (int c0 = 0; c0 < K; c0 += C) {
            if (!mb_wait(&rg.full[rg.slot], rg.ph, abort_flag, err, rg.lim)) return false;
            if (CB == kStepConsumerWarps || nr > 0) {  // one row block per slot: every warp has rows
                const uint8_t *sa = rg.buf + (size_t)rg.slot * kPiece + ((size_t)rb * C + cw) * 2;
                const float *xp = xs + c0 + cw;
                float4 x[STEPS];
                uint2 w[4][STEPS];
#pragma unroll
                for (int j = 0; j < STEPS; j++) {
                    x[j] = *reinterpret_cast<const float4 *>(xp + j * 128);
#pragma unroll
                    for (int r = 0; r < 4; r++)
                        w[r][j] = *reinterpret_cast<const uint2 *>(sa + (size_t)r * C * 2 + j * 256);
                }
                __syncwarp();
                if (lane == 0)
                    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&rg.empty[rg.slot])) : "memory");
#pragma unroll
                for (int j = 0; j < STEPS; j++)
#pragma unroll
                    for (int r = 0; r < 4; r++) p[r][j] = dot4(w[r][j], x[j], p[r][j]);
            } else if (lane == 0) {
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&rg.empty[rg.slot])) : "memory");
            }
            if (++rg.slot == kRing) { rg.slot = 0; rg.ph ^= 1u; }
        }
        if (CB != kStepConsumerWarps && nr <= 0) continue;
        float t[4];
#pragma unroll
        for (int r = 0; r < 4; r++) {
            t[r] = 0.f;
#pragma unroll
            for (int j = 0; j < STEPS; j++) t[r] += p[r][j];
        }
        const float tot = warp_sum4(t[0], t[1], t[2], t[3]);
        if ((lane & 7) == 0 && (lane >> 3) < nr) {
            float *dst = acc + (ra - r0) + rb + (lane >> 3);
            if (CB == 1) *dst += tot;  // one warp per row: no other writer
            else atomicAdd(dst, tot);
        }
    }
    return true;
}

// ---- the 4-row ring of the tp = 1 kernel: every slot holds 4 rows of up to 4096 columns ----
// (the tensor-parallel kernel uses the rows x columns slots above, whose narrow shards need them)
__device__ __forceinline__ bool produce_r4(Ring &rg, const __nv_bfloat16 *W, int N, int K, volatile int *abort_flag,
                                        int *err, uint32_t &issued, uint32_t &last_ph, uint64_t policy) {
    int r0, r1;
    split_rows(N, blockIdx.x, gridDim.x, r0, r1);
    const int C = chunk_cols(K);
    for (int ra = r0; ra < r1; ra += 4) {
        const int nr = min(4, r1 - ra);
        for (int c0 = 0; c0 < K; c0 += C) {
            if (!mb_wait(&rg.empty[rg.slot], rg.ph ^ 1u, abort_flag, err, rg.lim)) return false;
            const uint32_t fb = su32(&rg.full[rg.slot]);
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(fb), "r"((uint32_t)(nr * C * 2))
                         : "memory");
            for (int j = 0; j < nr; j++)
                asm volatile(
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
                    "%4;" ::"r"(su32(rg.buf + (size_t)rg.slot * kPiece + (size_t)j * C * 2)),
                    "l"(W + (size_t)(ra + j) * K + c0), "r"((uint32_t)(C * 2)), "r"(fb), "l"(policy)
                    : "memory");
            issued |= 1u << rg.slot;
            last_ph = (last_ph & ~(1u << rg.slot)) | (rg.ph << rg.slot);
            if (++rg.slot == kRing) { rg.slot = 0; rg.ph ^= 1u; }
        }
    }
    return true;
}

template <int C>
__device__ __forceinline__ bool consume_c_r4(Ring &rg, int K, const float *xs, float *acc, int r0, int r1,
                                          volatile int *abort_flag, int *err) {
    constexpr int PER_WARP = C / 8;
    constexpr int STEPS = PER_WARP / 128;
    static_assert(STEPS >= 1, "C >= 1024 (see consume_512)");
    static_assert(4 == 4, "warp_sum4 reduces four rows");
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int cw = warp * PER_WARP + lane * 4;
    for (int ra = r0; ra < r1; ra += 4) {
        const int nr = min(4, r1 - ra);
        float p[4][STEPS];
#pragma unroll
        for (int r = 0; r < 4; r++)
#pragma unroll
            for (int j = 0; j < STEPS; j++) p[r][j] = 0.f;
        for (int c0 = 0; c0 < K; c0 += C) {
            if (!mb_wait(&rg.full[rg.slot], rg.ph, abort_flag, err, rg.lim)) return false;
            const uint8_t *sa = rg.buf + (size_t)rg.slot * kPiece + (size_t)cw * 2;
            const float *xp = xs + c0 + cw;
            float4 x[STEPS];
            uint2 w[4][STEPS];
#pragma unroll
            for (int j = 0; j < STEPS; j++) {
                x[j] = *reinterpret_cast<const float4 *>(xp + j * 128);
#pragma unroll
                for (int r = 0; r < 4; r++)
                    w[r][j] = *reinterpret_cast<const uint2 *>(sa + (size_t)r * C * 2 + j * 256);
            }
            __syncwarp();
            if (lane == 0)
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&rg.empty[rg.slot])) : "memory");
            if (++rg.slot == kRing) { rg.slot = 0; rg.ph ^= 1u; }
#pragma unroll
            for (int j = 0; j < STEPS; j++)
#pragma unroll
                for (int r = 0; r < 4; r++) p[r][j] = dot4(w[r][j], x[j], p[r][j]);
        }
        float t[4];
#pragma unroll
        for (int r = 0; r < 4; r++) {
            t[r] = 0.f;
#pragma unroll
            for (int j = 0; j < STEPS; j++) t[r] += p[r][j];
        }
        const float tot = warp_sum4(t[0], t[1], t[2], t[3]);
        if ((lane & 7) == 0 && (lane >> 3) < nr) atomicAdd(acc + (ra - r0) + (lane >> 3), tot);
    }
    return true;
}

// C = 512 (K an odd multiple of 512, e.g. a tensor-parallel shard): warp w takes 64 columns of each
// slot, lane l columns 2l, 2l+1
__device__ __forceinline__ bool consume_512_r4(Ring &rg, int K, const float *xs, float *acc, int r0, int r1,
                                            volatile int *abort_flag, int *err) {
    constexpr int C = 512;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int cw = warp * 64 + lane * 2;
    for (int ra = r0; ra < r1; ra += 4) {
        const int nr = min(4, r1 - ra);
        float p[4] = {0.f, 0.f, 0.f, 0.f};
        for (int c0 = 0; c0 < K; c0 += C) {
            if (!mb_wait(&rg.full[rg.slot], rg.ph, abort_flag, err, rg.lim)) return false;
            const uint8_t *sa = rg.buf + (size_t)rg.slot * kPiece + (size_t)cw * 2;
            const float2 x = *reinterpret_cast<const float2 *>(xs + c0 + cw);
            uint32_t w[4];
#pragma unroll
            for (int r = 0; r < 4; r++) w[r] = *reinterpret_cast<const uint32_t *>(sa + (size_t)r * C * 2);
            __syncwarp();
            if (lane == 0)
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&rg.empty[rg.slot])) : "memory");
            if (++rg.slot == kRing) { rg.slot = 0; rg.ph ^= 1u; }
#pragma unroll
            for (int r = 0; r < 4; r++) p[r] = fmaf(bf16hi(w[r]), x.y, fmaf(bf16lo(w[r]), x.x, p[r]));
        }
        const float tot = warp_sum4(p[0], p[1], p[2], p[3]);
        if ((lane & 7) == 0 && (lane >> 3) < nr) atomicAdd(acc + (ra - r0) + (lane >> 3), tot);
    }
    return true;
}

__device__ __forceinline__ bool consume_r4(Ring &rg, int N, int K, const float *xs, float *acc, int &r0, int &r1,
                                        volatile int *abort_flag, int *err) {
    split_rows(N, blockIdx.x, gridDim.x, r0, r1);
    const int tid = threadIdx.x;
    for (int r = tid; r < r1 - r0; r += kStepConsumers) acc[r] = 0.f;
    consumers_sync();
    bool ok;
    switch (chunk_cols(K)) {
        case 4096: ok = consume_c_r4<4096>(rg, K, xs, acc, r0, r1, abort_flag, err); break;
        case 2048: ok = consume_c_r4<2048>(rg, K, xs, acc, r0, r1, abort_flag, err); break;
        case 1024: ok = consume_c_r4<1024>(rg, K, xs, acc, r0, r1, abort_flag, err); break;
        default: ok = consume_512_r4(rg, K, xs, acc, r0, r1, abort_flag, err); break;
    }
    if (!ok) return false;
    consumers_sync();
    return true;
}

// every CTA's writes before the barrier are visible to every CTA after it

template <int C>
__device__ __forceinline__ bool consume_narrow(Ring &rg, int K, const float *xs, float *acc, int r0, int r1,
                                            volatile int *abort_flag, int *err) {
    return consume_c<C>(rg, K, xs, acc, r0, r1, abort_flag, err);
}

__device__ __forceinline__ bool consume(Ring &rg, int N, int K, const float *xs, float *acc, int &r0, int &r1,
                                        volatile int *abort_flag, int *err) {
    split_rows(N, blockIdx.x, gridDim.x, r0, r1);
    const int tid = threadIdx.x;
    for (int r = tid; r < r1 - r0; r += kStepConsumers) acc[r] = 0.f;
    consumers_sync();
    bool ok;
    switch (chunk_cols(K)) {
        case 4096: ok = consume_c<4096>(rg, K, xs, acc, r0, r1, abort_flag, err); break;
        case 2048: ok = consume_narrow<2048>(rg, K, xs, acc, r0, r1, abort_flag, err); break;
        case 1024: ok = consume_narrow<1024>(rg, K, xs, acc, r0, r1, abort_flag, err); break;
        default: ok = consume_narrow<512>(rg, K, xs, acc, r0, r1, abort_flag, err); break;
    }
    if (!ok) return false;
    consumers_sync();
    return true;
}

// This CTA's arrival at a barrier: one release-add on the grid's counter.  The test hook a.stall_cta makes
// one CTA withhold its arrival at the step's first barrier, so that every wait on it runs out.
__device__ __forceinline__ void arrive(const StepArgs &a, unsigned idx) {
    if (idx == 0 && (int)blockIdx.x == a.stall_cta) return;
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.bar) : "memory");
}

// every CTA's writes before the barrier are visible to every CTA after it
__device__ __forceinline__ bool grid_sync(const StepArgs &a, unsigned &target, volatile int *abort_flag) {
    consumers_sync();
    const unsigned idx = target / gridDim.x;
    target += gridDim.x;
    if (threadIdx.x == 0 && a.trace && blockIdx.x == 0) a.trace[2 * idx + 1] = trace_ns();
    if (threadIdx.x == 0) {
        // release: this CTA's writes (ordered before by the named barrier above) are visible to whoever acquires
        // the count; the acquire polls order every later read after the other CTAs' writes
        arrive(a, idx);
        const uint64_t t0 = now_ns();
        while (ld_acquire(a.bar) < target) {
            if (*abort_flag || ld_acquire(reinterpret_cast<unsigned *>(a.err)) != 0u) { *abort_flag = 1; break; }
            if (now_ns() - t0 > a.wait_cycles) {
                *abort_flag = 1;
                atomicExch(a.err, 2);
                break;
            }
        }
        if (a.trace && blockIdx.x == 0) a.trace[2 * idx + 2] = trace_ns();
    }
    consumers_sync();
    return !*abort_flag;
}

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// ---- tensor-parallel exchanges: flag-in-data words over NVLink, no fences ----
// Every value a rank sends travels as one 8-byte word (fp32 bits | generation << 32), written with one
// 64-bit store into the receiver's inbox and read with 64-bit loads: the store is single-copy atomic, so a
// word that shows this exchange's generation carries this exchange's value, and the receiver needs no
// barrier or fence to trust it.  Generations grow by one per exchange (identically on every rank, and
// across steps through a.gen), so a slot never shows a stale word with the current generation.
__device__ __forceinline__ unsigned long long ll_pack(float v, unsigned gen) {
    return (unsigned long long)__float_as_uint(v) | ((unsigned long long)gen << 32);
}
__device__ __forceinline__ void st_ll(unsigned *p, unsigned long long w) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_ll(const unsigned *p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
// Wait (bounded) for the word at p to carry generation gen; its value, or false on expiry.
__device__ __forceinline__ bool wait_ll(const StepArgs &a, const unsigned *p, unsigned gen, float &v,
                                        volatile int *abort_flag) {
    unsigned long long w = ld_ll(p);
    if ((unsigned)(w >> 32) != gen) {
        const uint64_t t0 = now_ns();
        do {
            if (*abort_flag || now_ns() - t0 > a.wait_cycles) return false;
            w = ld_ll(p);
        } while ((unsigned)(w >> 32) != gen);
    }
    v = __uint_as_float((unsigned)w);
    return true;
}

// this rank's partial of rows [r0, r1) of a row-split projection (O, down) into slot `rank` of every rank's
// inbox `box` ([tp][D] words of 8 bytes)
__device__ __forceinline__ void push_ll(const StepArgs &a, int box, int r0, int r1, const float *acc, unsigned gen) {
    const int n = (r1 - r0) * a.tp;
    for (int i = threadIdx.x; i < n; i += kStepConsumers) {
        const int r = i / a.tp, p = i % a.tp;
        st_ll(a.xch[p] + box + 2 * ((size_t)a.rank * a.D + r0 + r), ll_pack(acc[r], gen));
    }
}

// The all-reduce of rows [r0, r1) (this CTA's rows of the projection): wait for every rank's partial of
// them in this rank's inbox and add them, in rank order (the same sum on every rank), into the residual
// stream x.  A grid barrier follows before any CTA reads x.
__device__ __forceinline__ bool reduce_ll(const StepArgs &a, int box, int r0, int r1, float *x, unsigned gen,
                                          float *scratch, volatile int *abort_flag, int *fail) {
    const int n = (r1 - r0) * a.tp;
    const unsigned *in = a.xch[a.rank] + box;
    for (int i = threadIdx.x; i < n; i += kStepConsumers) {
        const int r = i / a.tp, p = i % a.tp;
        float v = 0.f;
        if (!wait_ll(a, in + 2 * ((size_t)p * a.D + r0 + r), gen, v, abort_flag)) *fail = 1;
        scratch[i] = v;
    }
    consumers_sync();
    if (*fail) {
        if (threadIdx.x == 0) {
            *abort_flag = 1;
            atomicExch(a.err, 4);
        }
        return false;
    }
    for (int r = threadIdx.x; r < r1 - r0; r += kStepConsumers) {
        float t = __ldcg(x + r0 + r);
        for (int p = 0; p < a.tp; p++) t += scratch[r * a.tp + p];
        x[r0 + r] = t;
    }
    return true;
}

// CTA 0 sends this rank's q / k sums of squares of the layer (complete after the QKV grid barrier) to every
// rank: slot `rank` of their kXSs inbox ([tp][2] words)
__device__ __forceinline__ void push_ss(const StepArgs &a, int layer, unsigned gen) {
    if (blockIdx.x != 0 || threadIdx.x >= a.tp) return;
    const float sq = __ldcg(a.ss + 2 * layer), sk = __ldcg(a.ss + 2 * layer + 1);
    unsigned *dst = a.xch[threadIdx.x] + kXSs + 4 * a.rank;
    st_ll(dst, ll_pack(sq, gen));
    st_ll(dst + 2, ll_pack(sk, gen));
}

// xs = rmsnorm(src) * w over K elements (src read through L2); with w == nullptr a plain copy.
// Loads are issued in batches of 4 float4 per thread so that their L2 latencies overlap.
__device__ __forceinline__ void load_vec(float *xs, const float *src, int K, const float *w, float eps, float *red) {
    const int tid = threadIdx.x;
    const int n4 = K >> 2;
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
    float4 *x4 = reinterpret_cast<float4 *>(xs);
    float ss = 0.f;
    for (int b = 0; b < n4; b += 4 * kStepConsumers) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int q = b + u * kStepConsumers + tid;
            v[u] = q < n4 ? __ldcg(s4 + q) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int q = b + u * kStepConsumers + tid;
            if (q < n4) x4[q] = v[u];
            ss += v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
        }
    }
    if (!w) { consumers_sync(); return; }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    consumers_sync();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kStepConsumerWarps; i++) tot += red[i];
    const float sc = 1.0f / sqrtf(tot / (float)K + eps);
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
    for (int q = tid; q < n4; q += kStepConsumers) {
        float4 v = x4[q];
        const float4 g = w4[q];
        v.x = g.x * v.x * sc; v.y = g.y * v.y * sc; v.z = g.z * v.z * sc; v.w = g.w * v.w * sc;
        x4[q] = v;
    }
    consumers_sync();
}

// xs[p] = up[p] * silu(gate[p]) for the (2F) gate/up outputs, rows interleaved in blocks of 16
// (kGuBlock) gate rows then the 16 matching up rows; float4-wide, loads batched.
__device__ __forceinline__ void load_swiglu(float *xs, const float *gu, int F) {
    const int tid = threadIdx.x;
    const int n4 = F >> 2;  // float4 outputs
    float4 *x4 = reinterpret_cast<float4 *>(xs);
    for (int b = 0; b < n4; b += 4 * kStepConsumers) {
        float4 g[4], u[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int q = b + k * kStepConsumers + tid;
            if (q < n4) {
                const int blk = q >> 2, off = (q & 3) * 4;
                g[k] = __ldcg(reinterpret_cast<const float4 *>(gu + (size_t)blk * 2 * kGuBlock + off));
                u[k] = __ldcg(reinterpret_cast<const float4 *>(gu + (size_t)blk * 2 * kGuBlock + kGuBlock + off));
            }
        }
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int q = b + k * kStepConsumers + tid;
            if (q < n4) {
                float4 h;
                h.x = u[k].x * (g[k].x * (1.0f / (1.0f + expf(-g[k].x))));
                h.y = u[k].y * (g[k].y * (1.0f / (1.0f + expf(-g[k].y))));
                h.z = u[k].z * (g[k].z * (1.0f / (1.0f + expf(-g[k].z))));
                h.w = u[k].w * (g[k].w * (1.0f / (1.0f + expf(-g[k].w))));
                x4[q] = h;
            }
        }
    }
    consumers_sync();
}

template <typename KT, int DPL> struct SKV;
template <> struct SKV<__nv_bfloat16, 4> {
    using T = uint2;
    static __device__ __forceinline__ T load(const __nv_bfloat16 *p) { return *reinterpret_cast<const uint2 *>(p); }
    static __device__ __forceinline__ void unpack(const T &u, float *f) {
        f[0] = bf16lo(u.x); f[1] = bf16hi(u.x); f[2] = bf16lo(u.y); f[3] = bf16hi(u.y);
    }
};
template <> struct SKV<__nv_bfloat16, 2> {
    using T = uint32_t;
    static __device__ __forceinline__ T load(const __nv_bfloat16 *p) { return *reinterpret_cast<const uint32_t *>(p); }
    static __device__ __forceinline__ void unpack(const T &u, float *f) { f[0] = bf16lo(u); f[1] = bf16hi(u); }
};
template <> struct SKV<float, 4> {
    using T = float4;
    static __device__ __forceinline__ T load(const float *p) { return *reinterpret_cast<const float4 *>(p); }
    static __device__ __forceinline__ void unpack(const T &u, float *f) { f[0] = u.x; f[1] = u.y; f[2] = u.z; f[3] = u.w; }
};
template <> struct SKV<float, 2> {
    using T = float2;
    static __device__ __forceinline__ T load(const float *p) { return *reinterpret_cast<const float2 *>(p); }
    static __device__ __forceinline__ void unpack(const T &u, float *f) { f[0] = u.x; f[1] = u.y; }
};

// Keys of an attention item's first tile staged into shared memory during the QKV phase.
template <typename KT>
__host__ __device__ constexpr int stage_keys() { return sizeof(KT) == 2 ? 64 : 32; }

// Issue cp.async copies of the cached K and V rows [t0, t0 + stage_keys) (except the current
// position, computed in this step) of KV head kvh into `stage`: K rows, then V rows.
template <typename KT, int D>
__device__ __forceinline__ void stage_kv(const StepArgs &a, const StepLayer &Ly, int kvh, int t0, int t1, int pos,
                                         KT *stage) {
    constexpr int SK = stage_keys<KT>();
    constexpr int CH = D * (int)sizeof(KT) / 16;  // 16-byte chunks per row
    const int nrows = min(SK, t1 - t0);
    const int *ptab = a.page_table + (size_t)(a.slots ? *a.slots : 0) * a.max_pages;
    const int ps = a.page_size, lg = a.log2_page;
    for (int i = threadIdx.x; i < 2 * nrows * CH; i += kStepConsumers) {
        const int which = i / (nrows * CH), rem = i % (nrows * CH), r = rem / CH, c = rem % CH;
        const int tt = t0 + r;
        if (tt == pos) continue;
        const KT *cache = reinterpret_cast<const KT *>(which ? Ly.vc : Ly.kc);
        const KT *src = cache + (((size_t)ptab[tt >> lg] * a.Hkv + kvh) * ps + (tt & (ps - 1))) * D + c * (16 / sizeof(KT));
        const uint32_t dst = su32(stage + (size_t)(which * SK + r) * D) + c * 16;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// One attention work item (KV head kvh, context split sp of ns): QK-norm + RoPE of its query heads
// and key, the KV-cache write (split 0), online-softmax attention over its keys, partial or final
// output, and the merge of all splits by the last CTA to finish this KV head.  The whole-vector
// QK-norm uses the sums of squares the QKV phase accumulated (a.ss).
// 2^x by the hardware approximation (ex2.approx, flushes subnormals): attention scores are kept in the
// log2 domain (the scale carries log2 e), the usual flash-attention formulation
__device__ __forceinline__ float exp2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// sub-phase timestamps of CTA 0's attention item (profiling runs only): slot k of layer `layer`,
// after the per-phase pairs
__device__ __forceinline__ void attn_mark(const StepArgs &a, int layer, int k) {
    if (a.trace && blockIdx.x == 0 && threadIdx.x == 0)
        a.trace[2 * (5 * a.layers + 1) + (size_t)layer * 8 + k] = trace_ns();
}

template <typename KT, int D, int G, bool TPM>
__device__ void attn_item(const StepArgs &a, const StepLayer &Ly, int layer, int kvh, int sp, int ns, float *sm,
                          const KT *stage, unsigned ss_gen, volatile int *abort_flag) {
    constexpr int DPL = D / 32;
    constexpr int HALF = D / 2;
    using KV = SKV<KT, DPL>;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float *qs = sm;                 // [G][D]
    float *ks = qs + G * D;         // [D]
    float *vs = ks + D;             // [D]
    float *wo = vs + D;             // [4][G][D]  warp partials, merged in two rounds
    float *wm = wo + 4 * G * D;     // [8][G]
    float *wl = wm + 8 * G;         // [8][G]
    float *mlm = wl + 8 * G;        // [G][64] split maxima, then weights
    float *mll = mlm + G * 64;      // [G][64] split sums
    const int pos = *a.positions;
    const int n = pos + 1;
    const int chunk = (n + ns - 1) / ns;
    const int t0 = sp * chunk, t1 = min(n, t0 + chunk);
    const int Q = a.H * D, KVw = a.Hkv * D;
    // ---- q heads, k, v of this KV head (one float4 per thread for d 128, G 4) ----
    float scq = 1.f, sck = 1.f;
    if (a.qk_mode == 1) {
        float tq = 0.f, tk = 0.f;
        if constexpr (TPM) {  // every rank's sums (flag-in-data words), added in rank order: the same total on every rank
            __shared__ float ss_in[2 * 8];
            __shared__ int ss_fail;
            if (threadIdx.x == 0) ss_fail = 0;
            consumers_sync();
            if ((int)threadIdx.x < 2 * a.tp) {
                float v = 0.f;
                if (!wait_ll(a, a.xch[a.rank] + kXSs + 2 * threadIdx.x, ss_gen, v, abort_flag)) ss_fail = 1;
                ss_in[threadIdx.x] = v;
            }
            consumers_sync();
            if (ss_fail) {
                if (threadIdx.x == 0) {
                    *abort_flag = 1;
                    atomicExch(a.err, 4);
                }
                return;
            }
            for (int p = 0; p < a.tp; p++) {
                tq += ss_in[2 * p];
                tk += ss_in[2 * p + 1];
            }
        } else {
            tq = __ldcg(a.ss + 2 * layer);
            tk = __ldcg(a.ss + 2 * layer + 1);
        }
        scq = 1.0f / sqrtf(tq / (float)a.q_total + 1e-6f);
        sck = 1.0f / sqrtf(tk / (float)a.kv_total + 1e-6f);
    }
    constexpr int NQ4 = G * D / 4, NK4 = D / 4;
    attn_mark(a, layer, 0);
    asm volatile("cp.async.wait_all;" ::: "memory");  // this item's first key tile, staged during the QKV phase
    for (int i = tid; i < NQ4 + 2 * NK4; i += kStepConsumers) {
        float4 v;
        if (i < NQ4) {
            v = __ldcg(reinterpret_cast<const float4 *>(a.qkv + (size_t)kvh * G * D) + i);
            if (a.qk_mode == 1) {
                const float4 g = reinterpret_cast<const float4 *>(Ly.qn + (size_t)kvh * G * D)[i];
                v.x *= g.x * scq; v.y *= g.y * scq; v.z *= g.z * scq; v.w *= g.w * scq;
            }
            reinterpret_cast<float4 *>(qs)[i] = v;
        } else if (i < NQ4 + NK4) {
            v = __ldcg(reinterpret_cast<const float4 *>(a.qkv + Q + (size_t)kvh * D) + (i - NQ4));
            if (a.qk_mode == 1) {
                const float4 g = reinterpret_cast<const float4 *>(Ly.kn + (size_t)kvh * D)[i - NQ4];
                v.x *= g.x * sck; v.y *= g.y * sck; v.z *= g.z * sck; v.w *= g.w * sck;
            }
            reinterpret_cast<float4 *>(ks)[i - NQ4] = v;
        } else {
            v = __ldcg(reinterpret_cast<const float4 *>(a.qkv + Q + KVw + (size_t)kvh * D) + (i - NQ4 - NK4));
            v.x = Elt<KT>::round(v.x); v.y = Elt<KT>::round(v.y); v.z = Elt<KT>::round(v.z); v.w = Elt<KT>::round(v.w);
            reinterpret_cast<float4 *>(vs)[i - NQ4 - NK4] = v;
        }
    }
    consumers_sync();
    attn_mark(a, layer, 1);
    if (a.qk_mode == 2) {
        for (int hh = warp; hh <= G; hh += 8) {
            float *v = hh < G ? qs + hh * D : ks;
            const float *w = hh < G ? Ly.qn + (size_t)(kvh * G + hh) * D : Ly.kn + (size_t)kvh * D;
            float s2 = 0.f;
            for (int i = lane; i < D; i += 32) s2 += v[i] * v[i];
            s2 = warp_sum(s2);
            const float sc = 1.0f / sqrtf(s2 / (float)D + 1e-6f);
            for (int i = lane; i < D; i += 32) v[i] = w[i] * v[i] * sc;
        }
        consumers_sync();
    }
    // ---- RoPE (split-half) of the G query heads and the key; the key is rounded to the cache type ----
    const int *ptab = a.page_table + (size_t)(a.slots ? *a.slots : 0) * a.max_pages;
    KT *kc = reinterpret_cast<KT *>(Ly.kc);
    KT *vc = reinterpret_cast<KT *>(Ly.vc);
    const int ps = a.page_size, lg = a.log2_page, Hkv = a.Hkv;
    const size_t cbase = (((size_t)ptab[pos >> lg] * Hkv + kvh) * ps + (pos & (ps - 1))) * D;
    const float2 *fr = a.freq + (size_t)pos * HALF;
    for (int i = tid; i < (G + 1) * HALF; i += kStepConsumers) {
        const int hh = i / HALF, f = i % HALF;
        float *v = hh < G ? qs + hh * D : ks;
        const float2 cs = fr[f];
        const float x1 = v[f], x2 = v[f + HALF];
        float y1 = x1 * cs.x - x2 * cs.y, y2 = x2 * cs.x + x1 * cs.y;
        if (hh == G) {
            y1 = Elt<KT>::round(y1);
            y2 = Elt<KT>::round(y2);
            if (sp == 0) {
                Elt<KT>::store(kc + cbase + f, y1);
                Elt<KT>::store(kc + cbase + f + HALF, y2);
            }
        }
        v[f] = y1;
        v[f + HALF] = y2;
    }
    if (sp == 0)
        for (int i = tid; i < D; i += kStepConsumers) Elt<KT>::store(vc + cbase + i, vs[i]);
    consumers_sync();
    attn_mark(a, layer, 2);
    // ---- keys [t0, t1): warp w takes keys t0 + 64 j + 8 w .. + 7 ----
    float qreg[G][DPL];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int j = 0; j < DPL; j++) qreg[g][j] = qs[g * D + lane * DPL + j] * (a.scale * 1.4426950408889634f);
    float m[G], l[G], o[G][DPL];
#pragma unroll
    for (int g = 0; g < G; g++) {
        m[g] = -INFINITY; l[g] = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; j++) o[g][j] = 0.f;
    }
    for (int tb = t0; tb < t1; tb += 8 * kStepTPW) {
        typename KV::T kr[kStepTPW], vr[kStepTPW];
#pragma unroll
        for (int j = 0; j < kStepTPW; j++) {
            const int tt = tb + warp * kStepTPW + j;
            if (tt < t1 && tt != pos) {
                if (tt < t0 + stage_keys<KT>()) {
                    kr[j] = KV::load(stage + (size_t)(tt - t0) * D + lane * DPL);
                    vr[j] = KV::load(stage + (size_t)(stage_keys<KT>() + tt - t0) * D + lane * DPL);
                } else {
                    const size_t base = (((size_t)ptab[tt >> lg] * Hkv + kvh) * ps + (tt & (ps - 1))) * D + lane * DPL;
                    kr[j] = KV::load(kc + base);
                    vr[j] = KV::load(vc + base);
                }
            }
        }
        float sc[kStepTPW][G];
#pragma unroll
        for (int j = 0; j < kStepTPW; j++) {
            const int tt = tb + warp * kStepTPW + j;
            float kf[DPL];
            if (tt == pos) {
#pragma unroll
                for (int e = 0; e < DPL; e++) kf[e] = ks[lane * DPL + e];
            } else if (tt < t1) {
                KV::unpack(kr[j], kf);
            } else {
#pragma unroll
                for (int e = 0; e < DPL; e++) kf[e] = 0.f;
            }
#pragma unroll
            for (int g = 0; g < G; g++) {
                float sdot = 0.f;
#pragma unroll
                for (int e = 0; e < DPL; e++) sdot = fmaf(qreg[g][e], kf[e], sdot);
                sc[j][g] = sdot;
            }
        }
        // reduce the lane-split dot products: the 8 x G sums share the shuffle levels
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
#pragma unroll
            for (int j = 0; j < kStepTPW; j++)
#pragma unroll
                for (int g = 0; g < G; g++) sc[j][g] += __shfl_xor_sync(0xffffffffu, sc[j][g], off);
#pragma unroll
        for (int j = 0; j < kStepTPW; j++)
            if (tb + warp * kStepTPW + j >= t1)
#pragma unroll
                for (int g = 0; g < G; g++) sc[j][g] = -INFINITY;
#pragma unroll
        for (int g = 0; g < G; g++) {
            float mx = m[g];
#pragma unroll
            for (int j = 0; j < kStepTPW; j++) mx = fmaxf(mx, sc[j][g]);
            if (mx == -INFINITY) continue;
            const float al = exp2_approx(m[g] - mx);
            l[g] *= al;
#pragma unroll
            for (int e = 0; e < DPL; e++) o[g][e] *= al;
            m[g] = mx;
#pragma unroll
            for (int j = 0; j < kStepTPW; j++) sc[j][g] = exp2_approx(sc[j][g] - mx);
        }
#pragma unroll
        for (int j = 0; j < kStepTPW; j++) {
            const int tt = tb + warp * kStepTPW + j;
            if (tt >= t1) continue;
            float vf[DPL];
            if (tt == pos) {
#pragma unroll
                for (int e = 0; e < DPL; e++) vf[e] = vs[lane * DPL + e];
            } else {
                KV::unpack(vr[j], vf);
            }
#pragma unroll
            for (int g = 0; g < G; g++) {
                l[g] += sc[j][g];
#pragma unroll
                for (int e = 0; e < DPL; e++) o[g][e] = fmaf(sc[j][g], vf[e], o[g][e]);
            }
        }
    }
    attn_mark(a, layer, 3);
    // ---- merge the 8 warps: warps 4..7 into warps 0..3, then the 4 through shared memory ----
    if (warp >= 4) {
#pragma unroll
        for (int g = 0; g < G; g++) {
            if (lane == 0) { wm[(warp - 4) * G + g] = m[g]; wl[(warp - 4) * G + g] = l[g]; }
#pragma unroll
            for (int j = 0; j < DPL; j++) wo[((warp - 4) * G + g) * D + lane * DPL + j] = o[g][j];
        }
    }
    consumers_sync();
    if (warp < 4) {
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float om = wm[warp * G + g], ol = wl[warp * G + g];
            const float M = fmaxf(m[g], om);
            const float ea = m[g] == -INFINITY ? 0.f : exp2_approx(m[g] - M);
            const float eb = om == -INFINITY ? 0.f : exp2_approx(om - M);
            l[g] = l[g] * ea + ol * eb;
#pragma unroll
            for (int j = 0; j < DPL; j++) o[g][j] = o[g][j] * ea + wo[(warp * G + g) * D + lane * DPL + j] * eb;
            m[g] = M;
        }
    }
    consumers_sync();
    if (warp < 4) {
#pragma unroll
        for (int g = 0; g < G; g++) {
            if (lane == 0) { wm[warp * G + g] = m[g]; wl[warp * G + g] = l[g]; }
#pragma unroll
            for (int j = 0; j < DPL; j++) wo[(warp * G + g) * D + lane * DPL + j] = o[g][j];
        }
    }
    consumers_sync();
    for (int i = tid; i < G * D; i += kStepConsumers) {
        const int g = i / D, j = i % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; w++) M = fmaxf(M, wm[w * G + g]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < 4; w++) {
                const float e = exp2_approx(wm[w * G + g] - M);
                L += wl[w * G + g] * e;
                O += wo[(w * G + g) * D + j] * e;
            }
        }
        const int h = kvh * G + g;
        if (ns == 1) {
            a.attn[(size_t)h * D + j] = O / L;
        } else {
            const size_t pidx = (size_t)h * ns + sp;
            a.part_o[pidx * D + j] = O;
            if (j == 0) { a.part_ml[pidx * 2] = M; a.part_ml[pidx * 2 + 1] = L; }
        }
    }
    if (ns == 1) return;
    // ---- every split CTA of this KV head waits for all partials, then merges its slice of the output ----
    consumers_sync();
    attn_mark(a, layer, 4);
    unsigned *cnt = a.counters + (size_t)layer * a.Hkv + kvh;  // zeroed before the launch
    if (tid == 0) {
        // release-add: the partials written above (ordered by the named barrier) are visible to the acquirers
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(cnt) : "memory");
        const uint64_t w0 = now_ns();
        while (ld_acquire(cnt) < (unsigned)ns) {
            if (now_ns() - w0 > a.wait_cycles) { atomicExch(a.err, 3); break; }
        }
    }
    consumers_sync();
    attn_mark(a, layer, 5);
    const int per = (G * D + ns - 1) / ns;
    const int i0 = sp * per, i1 = min(G * D, i0 + per);
    // the (max, sum) of every split of the heads this slice touches, and the slice's partial outputs,
    // loaded in one batch
    const int g0 = i0 / D, g1 = (i1 - 1) / D;
    for (int i = tid; i < (g1 - g0 + 1) * ns; i += kStepConsumers) {
        const int g = g0 + i / ns, sidx = i % ns;
        const float2 ml = __ldcg(reinterpret_cast<const float2 *>(a.part_ml) + (size_t)(kvh * G + g) * ns + sidx);
        mlm[g * 64 + sidx] = ml.x;
        mll[g * 64 + sidx] = ml.y;
    }
    constexpr int kMaxPV = 16;  // = the most splits attn_splits makes: one round of loads
    // outputs in rounds of one per thread; a round's loads of every split are issued together
    const int rounds = (i1 - i0 + kStepConsumers - 1) / kStepConsumers;
    float pv[kMaxPV];
    for (int rd = 0; rd < rounds; rd++) {
        const int oi = i0 + rd * kStepConsumers + tid;
        const bool mine = oi < i1;
        if (mine && ns <= kMaxPV) {
            const float *po = a.part_o + (size_t)(kvh * G + oi / D) * ns * D + oi % D;
#pragma unroll
            for (int sidx = 0; sidx < kMaxPV; sidx++) pv[sidx] = sidx < ns ? __ldcg(po + (size_t)sidx * D) : 0.f;
        }
        if (rd == 0) {
            consumers_sync();  // the (max, sum) loads above are in shared memory
            if (tid <= g1 - g0) {
                const int g = g0 + tid;
                float M = -INFINITY;
                for (int sidx = 0; sidx < ns; sidx++) M = fmaxf(M, mlm[g * 64 + sidx]);
                float L = 0.f;
                for (int sidx = 0; sidx < ns; sidx++) {
                    const float pm = mlm[g * 64 + sidx];
                    const float e = pm == -INFINITY ? 0.f : exp2_approx(pm - M);
                    L += mll[g * 64 + sidx] * e;
                    mlm[g * 64 + sidx] = e;
                }
                const float inv = 1.0f / L;
                for (int sidx = 0; sidx < ns; sidx++) mlm[g * 64 + sidx] *= inv;
            }
            consumers_sync();
        }
        if (!mine) continue;
        const int g = oi / D;
        float O = 0.f;
        if (ns <= kMaxPV) {
#pragma unroll
            for (int sidx = 0; sidx < kMaxPV; sidx++)
                if (sidx < ns) O += mlm[g * 64 + sidx] * pv[sidx];
        } else {
            const float *po = a.part_o + (size_t)(kvh * G + g) * ns * D + oi % D;
            for (int sidx = 0; sidx < ns; sidx++) O += mlm[g * 64 + sidx] * __ldcg(po + (size_t)sidx * D);
        }
        a.attn[(size_t)kvh * G * D + oi] = O;
    }
}

template <bool TPM>
__device__ __forceinline__ bool produce_t(Ring &rg, const __nv_bfloat16 *W, int N, int K, volatile int *abort_flag,
                                          int *err, uint32_t &issued, uint32_t &last_ph, uint64_t policy) {
    if constexpr (TPM) return produce(rg, W, N, K, abort_flag, err, issued, last_ph, policy);
    else return produce_r4(rg, W, N, K, abort_flag, err, issued, last_ph, policy);
}
template <bool TPM>
__device__ __forceinline__ bool consume_t(Ring &rg, int N, int K, const float *xs, float *acc, int &r0, int &r1,
                                          volatile int *abort_flag, int *err) {
    if constexpr (TPM) return consume(rg, N, K, xs, acc, r0, r1, abort_flag, err);
    else return consume_r4(rg, N, K, xs, acc, r0, r1, abort_flag, err);
}

template <typename KT, int D, int G, bool TPM>
__global__ void __launch_bounds__(kStepThreads, 1) qw_step_kernel(const StepArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full_bar[kRing], empty_bar[kRing];
    __shared__ int abort_sh, xfail;
    __shared__ float red[kStepConsumerWarps], red2[kStepConsumerWarps];
    __shared__ float am_v[kStepConsumers];
    __shared__ int am_i[kStepConsumers];
    uint8_t *ring = smem;                                            // kRing * kPiece
    float *xs = reinterpret_cast<float *>(smem + kRing * kPiece);    // max K floats
    float *acc = xs + a.xs_floats;                                   // max rows per CTA
    float *scratch = xs;                                             // attention phase only
    KT *stage = reinterpret_cast<KT *>(xs + a.stage_off);            // staged keys of this CTA's attention item
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    volatile int *abort_flag = &abort_sh;
    if (tid == 0) {
        for (int i = 0; i < kRing; i++) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&full_bar[i])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(&empty_bar[i])), "r"(kStepConsumerWarps)
                         : "memory");
        }
        abort_sh = 0;
        xfail = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    Ring rg{full_bar, empty_bar, ring, 0, 0u, a.wait_cycles, a.row_copies};
    const int D_ = a.D, Q = a.H * D, KVw = a.Hkv * D, QKV = Q + 2 * KVw, F = a.F;

    if (warp == kStepConsumerWarps) {
        // ======================= producer =======================
        if (lane == 0) {
            uint32_t issued = 0, last_ph = 0;
            bool ok = true;
            // the weights are read once per step: evict them first, so that L2 keeps the kernel's code, the
            // KV cache and the activations (evict_normal when turned off)
            uint64_t policy;
            if (a.evict_first)
                asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
            else
                asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(policy));
            for (int l = 0; l < a.layers && ok; l++) {
                const StepLayer &Ly = a.L[l];
                ok = ok && produce_t<TPM>(rg, Ly.w_qkv, QKV, D_, abort_flag, a.err, issued, last_ph, policy);
                ok = ok && produce_t<TPM>(rg, Ly.w_o, D_, Q, abort_flag, a.err, issued, last_ph, policy);
                ok = ok && produce_t<TPM>(rg, Ly.w_gu, 2 * F, D_, abort_flag, a.err, issued, last_ph, policy);
                ok = ok && produce_t<TPM>(rg, Ly.w_down, D_, F, abort_flag, a.err, issued, last_ph, policy);
            }
            ok = ok && produce_t<TPM>(rg, a.lm, a.V, D_, abort_flag, a.err, issued, last_ph, policy);
            if (!ok) {
                for (int i = 0; i < kRing; i++)
                    if (issued >> i & 1u) {
                        const uint32_t addr = su32(&full_bar[i]);
                        const uint64_t t0 = now_ns();
                        while (!mb_try(addr, (last_ph >> i) & 1u) && now_ns() - t0 < a.wait_cycles) {
                        }
                    }
            }
        }
        return;
    }

    // ======================= consumers =======================
    unsigned target = 0;
    unsigned gen = TPM ? *a.gen : 0u;                 // cross-rank barriers passed (monotonic across steps)
    int r0, r1;
    const int token = *a.tokens;
    constexpr bool tpm = TPM;  // tensor parallel: compiled only into the tp > 1 variants
    const int box_o = kXRows, box_d = kXRows + 2 * a.tp * D_;  // inboxes of [tp][D] 8-byte words
    float *xcur = a.x;  // residual stream (updated in place by the owner of each row)
    if (a.trace && blockIdx.x == 0 && tid == 0) a.trace[0] = trace_ns();
    for (int l = 0; l < a.layers; l++) {
        const StepLayer &Ly = a.L[l];
        // ---- rmsnorm + QKV ----
        if (l == 0) {
            const __nv_bfloat16 *er = a.embed + (size_t)token * D_;
            for (int k = tid; k < D_; k += kStepConsumers) {
                const float v = __bfloat162float(er[k]);
                if (blockIdx.x == 0) xcur[k] = v;
                xs[k] = v;
            }
            consumers_sync();
            // normalise in place (load_vec reads through L2; here the row came from the table)
            float ss = 0.f;
            for (int k = tid; k < D_; k += kStepConsumers) ss += xs[k] * xs[k];
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
            consumers_sync();
            float tot = 0.f;
            for (int i = 0; i < kStepConsumerWarps; i++) tot += red[i];
            const float sc = 1.0f / sqrtf(tot / (float)D_ + a.eps);
            for (int k = tid; k < D_; k += kStepConsumers) xs[k] = Ly.rms_att[k] * xs[k] * sc;
            consumers_sync();
        } else {
            load_vec(xs, xcur, D_, Ly.rms_att, a.eps, red);
        }
        {
            // start fetching this CTA's attention keys now: they land behind the QKV weight stream
            const int n = *a.positions + 1;
            const int ns = attn_splits(gridDim.x, a.Hkv, n);
            if ((int)blockIdx.x < a.Hkv * ns) {
                const int kvh = blockIdx.x / ns, sp = blockIdx.x % ns;
                const int chunk = (n + ns - 1) / ns;
                const int t0 = sp * chunk, t1 = min(n, t0 + chunk);
                if (t0 < t1) stage_kv<KT, D>(a, Ly, kvh, t0, t1, n - 1, stage);
            }
        }
        if (!consume_t<TPM>(rg, QKV, D_, xs, acc, r0, r1, abort_flag, a.err)) break;
        {
            // the QKV rows, and the sums of squares of the q and k rows for the whole-vector QK-norm
            float sq = 0.f, sk = 0.f;
            for (int r = tid; r < r1 - r0; r += kStepConsumers) {
                const float v = acc[r] + (Ly.b_qkv ? Ly.b_qkv[r0 + r] : 0.f);
                a.qkv[r0 + r] = v;
                if (r0 + r < Q) sq += v * v;
                else if (r0 + r < Q + KVw) sk += v * v;
            }
            if (a.qk_mode == 1) {
                sq = warp_sum(sq);
                sk = warp_sum(sk);
                if (lane == 0) { red[warp] = sq; red2[warp] = sk; }
                consumers_sync();
                float tq = 0.f, tk = 0.f;
                for (int w = 0; w < kStepConsumerWarps; w++) { tq += red[w]; tk += red2[w]; }
                sq = tq;
                sk = tk;
                if (tid == 0) {
                    if (tq != 0.f) atomicAdd(a.ss + 2 * l, tq);
                    if (tk != 0.f) atomicAdd(a.ss + 2 * l + 1, tk);
                }
            }
            if (!grid_sync(a, target, abort_flag)) break;
            if (tpm && a.qk_mode == 1) push_ss(a, l, ++gen);  // the layer's sums, complete after the barrier
        }
        // ---- attention (this rank's heads) ----
        {
            const int n = *a.positions + 1;
            const int ns = attn_splits(gridDim.x, a.Hkv, n);
            if ((int)blockIdx.x < a.Hkv * ns)
                attn_item<KT, D, G, TPM>(a, Ly, l, blockIdx.x / ns, blockIdx.x % ns, ns, scratch, stage, gen, abort_flag);
        }
        if (!grid_sync(a, target, abort_flag)) break;
        // ---- O projection + residual (summed over ranks through the inboxes) ----
        load_vec(xs, a.attn, Q, nullptr, 0.f, red);
        if (!consume_t<TPM>(rg, D_, Q, xs, acc, r0, r1, abort_flag, a.err)) break;
        if (tpm) {  // all-reduce of this CTA's rows over the ranks, into the residual stream
            push_ll(a, box_o, r0, r1, acc, ++gen);
            if (!reduce_ll(a, box_o, r0, r1, xcur, gen, xs, abort_flag, &xfail)) break;
        } else {
            for (int r = tid; r < r1 - r0; r += kStepConsumers) xcur[r0 + r] = __ldcg(xcur + r0 + r) + acc[r];
        }
        if (!grid_sync(a, target, abort_flag)) break;
        load_vec(xs, xcur, D_, Ly.rms_ffn, a.eps, red);
        // ---- gate/up (raw) ----
        if (!consume_t<TPM>(rg, 2 * F, D_, xs, acc, r0, r1, abort_flag, a.err)) break;
        for (int r = tid; r < r1 - r0; r += kStepConsumers) a.gu[r0 + r] = acc[r];
        if (!grid_sync(a, target, abort_flag)) break;
        // ---- SwiGLU (rows interleaved 16 gate / 16 up) + down + residual ----
        load_swiglu(xs, a.gu, F);
        if (!consume_t<TPM>(rg, D_, F, xs, acc, r0, r1, abort_flag, a.err)) break;
        if (tpm) {
            push_ll(a, box_d, r0, r1, acc, ++gen);
            if (!reduce_ll(a, box_d, r0, r1, xcur, gen, xs, abort_flag, &xfail)) break;
        } else {
            for (int r = tid; r < r1 - r0; r += kStepConsumers) xcur[r0 + r] = __ldcg(xcur + r0 + r) + acc[r];
        }
        if (!grid_sync(a, target, abort_flag)) break;
    }
    if (*abort_flag) {
        asm volatile("cp.async.wait_all;" ::: "memory");  // staged attention keys still in flight
        return;
    }
    // ---- final rmsnorm + lm_head (this rank's vocabulary rows) + argmax ----
    load_vec(xs, xcur, D_, a.norm_final, a.eps, red);
    if (!consume_t<TPM>(rg, a.V, D_, xs, acc, r0, r1, abort_flag, a.err)) return;
    if (a.trace && blockIdx.x == 0 && tid == 0) a.trace[2 * (target / gridDim.x) + 1] = trace_ns();
    float bv = -FLT_MAX;
    int bi = INT_MAX;
    for (int r = tid; r < r1 - r0; r += kStepConsumers) {
        const float v = acc[r];
        if (a.logits) a.logits[r0 + r] = v;
        if (v > bv) { bv = v; bi = r0 + r; }
    }
    am_v[tid] = bv;
    am_i[tid] = bi;
    consumers_sync();
    if (tid < 32) {
        for (int i = tid + 32; i < kStepConsumers; i += 32)
            if (am_v[i] > bv || (am_v[i] == bv && am_i[i] < bi)) { bv = am_v[i]; bi = am_i[i]; }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (tid == 0) {
            a.am_val[blockIdx.x] = bv;
            a.am_idx[blockIdx.x] = bi + a.v0;
            __threadfence();
            atomicAdd(a.bar, 1u);
        }
    }
    // CTA 0 gathers every CTA's winner, then (tensor parallel) every rank's, and feeds the token back
    if (blockIdx.x != 0 || warp != 0) return;
    target += gridDim.x;
    bool ok = true;
    if (lane == 0) {
        const uint64_t t0 = now_ns();
        while (ld_acquire(a.bar) < target)
            if (now_ns() - t0 > a.wait_cycles) { ok = false; break; }
    }
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    __threadfence();
    bv = -FLT_MAX;
    bi = INT_MAX;
    for (int c = lane; c < (int)gridDim.x; c += 32) {
        const float v = __ldcg(a.am_val + c);
        const int i = __ldcg(a.am_idx + c);
        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (tpm) {
        // every rank's winner: lane p sends this rank's (value, index) into slot `rank` of rank p's array and
        // then its generation flag; then lanes 0..tp-1 wait for every rank's flag
        gen += 1u;
        if (ok && lane < a.tp) {
            unsigned *in = a.xch[lane] + kXAm + 2 * a.rank;
            in[0] = __float_as_uint(bv);
            in[1] = (unsigned)bi;
            st_release_sys(a.xch[lane] + kXFlags + a.rank, gen);
        }
        if (ok && lane < a.tp) {
            const unsigned *mine = a.xch[a.rank] + kXFlags + lane;
            const uint64_t t0 = now_ns();
            while ((int)(ld_acquire_sys(mine) - gen) < 0)
                if (now_ns() - t0 > a.wait_cycles) { ok = false; break; }
        }
        ok = __all_sync(0xffffffffu, ok);
        bv = -FLT_MAX;
        bi = INT_MAX;
        if (lane < a.tp) {
            const unsigned *in = a.xch[a.rank] + kXAm + 2 * lane;
            bv = __uint_as_float(__ldcg(in));
            bi = (int)__ldcg(in + 1);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
    }
    if (lane == 0) {
        if (!ok) {
            atomicExch(a.err, 5);
            return;
        }
        if (a.argmax_out) *a.argmax_out = bi;
        if (a.hist) a.hist[*a.positions + 1] = bi;
        if (a.advance) {
            *a.tokens = bi;
            *a.positions += 1;
        }
        if (TPM) *a.gen = gen;
    }
}

template <typename KT, int D, bool TPM>
const void *step_fn_g(int G) {
    switch (G) {
        case 1: return (const void *)qw_step_kernel<KT, D, 1, TPM>;
        case 2: return (const void *)qw_step_kernel<KT, D, 2, TPM>;
        case 4: return (const void *)qw_step_kernel<KT, D, 4, TPM>;
        case 6: return (const void *)qw_step_kernel<KT, D, 6, TPM>;
        case 7: return (const void *)qw_step_kernel<KT, D, 7, TPM>;
        case 8: return (const void *)qw_step_kernel<KT, D, 8, TPM>;
    }
    return nullptr;
}

}  // namespace
}  // namespace qw

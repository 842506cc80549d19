// qw_gemm.cu -- the projections of prefill and batched decode on the 5th-generation tensor
// cores: tcgen05.mma with the accumulator in tensor memory (TMEM), operands staged in
// 128-byte-swizzled shared memory by TMA (cp.async.bulk.tensor, no multicast).
//
// Stands in for the reference's dense layer (LayerFeatures.dense, domain/graph/src/main/java/
// org/almostrealism/layers/LayerFeatures.java:785-830: y = W x with W (out, in) row-major)
// applied to many rows at once, with the neighbouring element-wise work fused into the
// epilogue: bias (Qwen2.5 layout), the residual accumulation of SequentialBlock.accum
// (SequentialBlock.java:413-429) and the SwiGLU product of FeedForwardFeatures.java:147-156.
//
// Layout of one CTA (persistent, one per SM, 192 threads):
//   warp 0      TMA producer: for every k-block, one 128 x 64 tile of W and one BN x 64 tile
//               of X into a ring of S shared-memory stages (full / empty mbarriers);
//   warp 1      allocates 2*BN TMEM columns; one lane issues 4 tcgen05.mma (M=128, N=BN,
//               K=16) per stage and commits the stage back to the producer, then commits the
//               finished accumulator to the epilogue;
//   warps 2-5   epilogue: tcgen05.ld of their 32 TMEM lanes (= 32 output features), fused
//               epilogue, coalesced stores (consecutive features across a warp).
// Two accumulators in TMEM let the epilogue of tile i overlap the MMAs of tile i+1.
// Tiles are visited in groups of 8 token tiles so that the CTAs running at the same time share
// their W and X tiles in L2.
//
// Launched with programmatic dependent launch: the prologue (barriers, TMEM, descriptor prefetch)
// and the first S weight tiles overlap the end of the previous kernel in the stream; the
// activation tiles and the epilogue wait for it (griddepcontrol.wait).
//
// Every mbarrier wait is bounded (kTcuWaitCycles); on expiry the CTA records TC_DEVERR_TIMEOUT,
// lets its issued copies and MMAs land, frees its TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>
#include <float.h>
#include <limits.h>
#include <mutex>
#include <stdlib.h>

#include "qw_internal.cuh"
#include "qw_tc.h"
#include "qw_tc_util.cuh"

namespace qw {

namespace {

constexpr int kTcThreads = 192;
constexpr int kBM = 128, kBK = 64;
constexpr int kGroupT = 8;
constexpr int kTcSmemBudget = 196 * 1024;

__host__ __device__ constexpr uint32_t tc_idesc(int bn) { return tc_idesc_f16(kBM, bn); }
__host__ __device__ constexpr int tc_stage_bytes(int bn) { return (kBM + bn) * kBK * 2; }
__host__ __device__ constexpr int tc_stages(int bn) {
    return kTcSmemBudget / tc_stage_bytes(bn) > 8 ? 8 : kTcSmemBudget / tc_stage_bytes(bn);
}
__host__ __device__ constexpr int tc_smem_bytes(int bn) { return tc_stages(bn) * tc_stage_bytes(bn) + 1024 + 4096; }

struct TileCoord {
    int f0, t0, kb0, kb1, ks;
};

__device__ __forceinline__ TileCoord tile_coord(int tile, int nf, int nt, int nks, int nkb) {
    TileCoord c;
    c.ks = tile % nks;
    const int j = tile / nks;
    const int per_group = nf * kGroupT;
    const int g = j / per_group, r = j % per_group;
    const int t_in = min(kGroupT, nt - g * kGroupT);
    c.t0 = (g * kGroupT + r % t_in);
    c.f0 = (r / t_in) * kBM;
    c.kb0 = (int)(((long long)nkb * c.ks) / nks);
    c.kb1 = (int)(((long long)nkb * (c.ks + 1)) / nks);
    return c;
}

// Epilogue of 32 consecutive tokens t0 .. t0+nj-1 of feature f (this lane) from the tile's sums v[j].
// split: 0 = whole sums; 1 + ks = K range ks of an atomically accumulated split (bias with range 0 only).
template <int EPI>
__device__ __forceinline__ void tc_emit(const TcArgs &a, float (&v)[32], const TileCoord &c, int f, int q, int lane,
                                        int t0, int nj, int split, uint8_t *sStage) {
    if (EPI == TC_SWIGLU) {
        // up * silu(gate) for this warp's 16 pairs x 32 tokens, staged as [token][64 pairs] bf16
        // so that the 4 epilogue warps then write whole 128-byte rows
        uint16_t *stg = reinterpret_cast<uint16_t *>(sStage);
#pragma unroll
        for (int j = 0; j < 32; j++) {
            const float g = v[j];
            const float u = __shfl_down_sync(0xffffffffu, g, 16);
            if (lane < 16) {
                const float h = u * __fdividef(g, 1.0f + __expf(-g));
                stg[j * 64 + q * 16 + lane] = f2bf_bits(h);
            }
        }
        asm volatile("bar.sync 2, 128;" ::: "memory");
        {
            const int et = threadIdx.x - 64;  // 0..127 over the epilogue warps
            const int pair0 = c.f0 >> 1;
            const int npair = min(64, (a.M - c.f0) >> 1);
            __nv_bfloat16 *o = reinterpret_cast<__nv_bfloat16 *>(a.out);
#pragma unroll
            for (int k2 = 0; k2 < 2; k2++) {
                const int idx = et + k2 * 128;  // 256 chunks of 16 bytes: 32 rows x 8
                const int row = idx >> 3, ch = idx & 7;
                if (row < nj && ch * 8 < npair) {
                    const uint4 u = *reinterpret_cast<const uint4 *>(stg + row * 64 + ch * 8);
                    *reinterpret_cast<uint4 *>(o + (size_t)(t0 + row) * a.ld_out + pair0 + ch * 8) = u;
                }
            }
        }
        asm volatile("bar.sync 2, 128;" ::: "memory");
    } else if (EPI == TC_ARGMAX) {
        // logits (optional), then the first maximum of this warp's 32 features for each of the
        // 32 tokens: a transposing butterfly leaves token j's winner in lane j
        int id[32];
#pragma unroll
        for (int j = 0; j < 32; j++) {
            if (f >= a.M) v[j] = -FLT_MAX;
            id[j] = f < a.M ? f : INT_MAX;
        }
        if (a.out && f < a.M) {
            float *o = reinterpret_cast<float *>(a.out);
#pragma unroll
            for (int j = 0; j < 32; j++)
                if (j < nj) o[(size_t)(t0 + j) * a.ld_out + f] = v[j];
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int j = 0; j < o; j++) {
                const float sv = up ? v[j] : v[j + o], kv = up ? v[j + o] : v[j];
                const int si = up ? id[j] : id[j + o], ki = up ? id[j + o] : id[j];
                const float rv = __shfl_xor_sync(0xffffffffu, sv, o);
                const int ri = __shfl_xor_sync(0xffffffffu, si, o);
                const bool take = rv > kv || (rv == kv && ri < ki);
                v[j] = take ? rv : kv;
                id[j] = take ? ri : ki;
            }
        }
        if (lane < nj) {
            const size_t ci = (size_t)(t0 + lane) * a.ncand + (c.f0 >> 5) + q;
            a.cand_val[ci] = v[0];
            a.cand_idx[ci] = id[0];
        }
    } else if (f < a.M) {
        float *o = reinterpret_cast<float *>(a.out);
        const float bias = (a.bias && split <= 1) ? a.bias[f] : 0.f;
        if (split) {
#pragma unroll
            for (int j = 0; j < 32; j++)
                if (j < nj) atomicAdd(o + (size_t)(t0 + j) * a.ld_out + f, v[j] + bias);
        } else if (EPI == TC_RESID) {
            // all residual loads first (out may alias resid), then the stores
            float rv[32];
#pragma unroll
            for (int j = 0; j < 32; j++) rv[j] = j < nj ? a.resid[(size_t)(t0 + j) * a.ld_resid + f] : 0.f;
#pragma unroll
            for (int j = 0; j < 32; j++)
                if (j < nj) o[(size_t)(t0 + j) * a.ld_out + f] = rv[j] + v[j];
        } else {
#pragma unroll
            for (int j = 0; j < 32; j++)
                if (j < nj) o[(size_t)(t0 + j) * a.ld_out + f] = v[j] + bias;
        }
    }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
    qw_tc_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, const TcArgs a) {
    constexpr int S = tc_stages(BN);
    constexpr int A_BYTES = kBM * kBK * 2, B_BYTES = BN * kBK * 2;
    constexpr uint32_t TMEM_COLS = 2 * BN;
    constexpr uint32_t IDESC = tc_idesc(BN);
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[S], empty_bar[S], tfull_bar[2], tempty_bar[2], done_bar;
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;

    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *sA = smem;
    uint8_t *sB = smem + S * A_BYTES;
    uint8_t *sStage = smem + S * (A_BYTES + B_BYTES);  // SWIGLU epilogue: [32 tokens][64 pairs] bf16
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    volatile int *abort_flag = &abort_sh;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&tfull_bar[i], 1);
            mbar_init(&tempty_bar[i], 4);
        }
        mbar_init(&done_bar, 1);
        abort_sh = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmW) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmX) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_sh;
    griddep_launch_dependents();  // the next kernel's prologue (and weight loads) may start

    const int nf = (a.M + kBM - 1) / kBM, nt = (a.T + BN - 1) / BN, nks = a.ksplit;
    const int nkb = (a.K + kBK - 1) / kBK;
    const int total = nf * nt * nks;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int s = 0;
            uint32_t ph = 0, issued = 0, last_ph = 0;
            bool ok = true;
            // The weights do not depend on the previous kernel in the stream: the first S stages load
            // their W tiles before the programmatic-launch wait, their X tiles (the previous kernel's
            // output) after it, into the same stage barrier.
            bool waited = false;
            int npend = 0, pend_kb[S], pend_t0[S];
            auto flush = [&]() {
                griddep_wait();
                waited = true;
                for (int i = 0; i < npend; i++)
                    tma_load_2d(sB + i * B_BYTES, &tmX, &full_bar[i], pend_kb[i] * kBK, pend_t0[i] * BN);
            };
            for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
                const TileCoord c = tile_coord(tile, nf, nt, nks, nkb);
                for (int kb = c.kb0; kb < c.kb1; kb++) {
                    if (!mbar_wait(&empty_bar[s], ph ^ 1u, abort_flag, a.err)) { ok = false; break; }
                    mbar_arrive_expect_tx(&full_bar[s], A_BYTES + B_BYTES);
                    tma_load_2d(sA + s * A_BYTES, &tmW, &full_bar[s], kb * kBK, c.f0);
                    if (waited) {
                        tma_load_2d(sB + s * B_BYTES, &tmX, &full_bar[s], kb * kBK, c.t0 * BN);
                    } else {  // stages 0..S-1 of the first pass, in order
                        pend_kb[npend] = kb;
                        pend_t0[npend] = c.t0;
                        if (++npend == S) flush();
                    }
                    issued |= 1u << s;
                    last_ph = (last_ph & ~(1u << s)) | (ph << s);
                    if (++s == S) { s = 0; ph ^= 1u; }
                }
            }
            if (!waited) flush();
            if (!ok) {
                // let every issued copy land before the CTA's shared memory goes away
                for (int i = 0; i < S; i++)
                    if (issued >> i & 1u) {
                        const uint32_t addr = smem_u32(&full_bar[i]);
                        const uint64_t t0 = gtime_ns();
                        while (!mbar_try(addr, (last_ph >> i) & 1u) && gtime_ns() - t0 < kTcuWaitCycles) {
                        }
                    }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            int s = 0, it = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, it++) {
                const TileCoord c = tile_coord(tile, nf, nt, nks, nkb);
                const int acc = it & 1;
                const uint32_t aph = (uint32_t)(it >> 1) & 1u;
                if (!mbar_wait(&tempty_bar[acc], aph ^ 1u, abort_flag, a.err)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(acc * BN);
                for (int kb = c.kb0; kb < c.kb1; kb++) {
                    if (!mbar_wait(&full_bar[s], ph, abort_flag, a.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t ad = sw128_desc(smem_u32(sA + s * A_BYTES));
                    const uint64_t bd = sw128_desc(smem_u32(sB + s * B_BYTES));
#pragma unroll
                    for (int k = 0; k < kBK / 16; k++)
                        tc_mma(d, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), IDESC, (kb > c.kb0 || k > 0) ? 1u : 0u);
                    tc_commit(&empty_bar[s]);
                    if (++s == S) { s = 0; ph ^= 1u; }
                }
                if (ok) tc_commit(&tfull_bar[acc]);
            }
            // all MMAs of this CTA complete before the TMEM is freed
            tc_commit(&done_bar);
            const uint32_t addr = smem_u32(&done_bar);
            const uint64_t t0 = gtime_ns();
            while (!mbar_try(addr, 0) && gtime_ns() - t0 < kTcuWaitCycles) {
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        griddep_wait();  // resid and out may belong to the previous kernel in the stream
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        int it = 0;
        for (int tile = blockIdx.x; tile < total; tile += gridDim.x, it++) {
            const TileCoord c = tile_coord(tile, nf, nt, nks, nkb);
            const int acc = it & 1;
            const uint32_t aph = (uint32_t)(it >> 1) & 1u;
            if (!mbar_wait(&tfull_bar[acc], aph, abort_flag, a.err)) break;
            tc_fence_after();
            const int f = c.f0 + q * 32 + lane;
            const int tbase = c.t0 * BN;
            const int ncols = min(BN, a.T - tbase);
            for (int cc = 0; cc < ncols; cc += 32) {
                uint32_t r[32];
                tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + cc), r);
                const int nj = min(32, ncols - cc);
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
                tc_emit<EPI>(a, v, c, f, q, lane, tbase + cc, nj, nks > 1 ? 1 + c.ks : 0, sStage);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty_bar[acc]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

// ---------------------------------------------------------------------------------------------
// CTA-pair variant for prefill shapes (cta_group::2): a cluster of two CTAs on two SMs computes a
// 256-feature x 256-token tile with one tcgen05.mma stream (M = 256, N = 256) issued by the even CTA.
// Each CTA stages its own 128 rows of W and its own 128 tokens of X per k-block (32 KB, six or seven stages),
// so a stage carries half the X bytes of the one-CTA 128 x 256 tile and the ring is deeper, and each
// CTA's TMEM holds the sums of its 128 features for all 256 tokens.
//   full[s]   in the even CTA: one arrival (its producer's expect_tx of both CTAs' bytes); both CTAs'
//             TMA loads count their bytes on it (cta_group::2 form, no multicast);
//   empty[s]  in each CTA, signalled by the MMA commit to both CTAs of the pair;
//   tfull[i]  in each CTA, signalled by the commit after the tile's last k-block;
//   tempty[i] in the even CTA: 8 arrivals (the epilogue warps of both CTAs).
// ---------------------------------------------------------------------------------------------
constexpr int kPairBM = 256, kPairBN = 256, kPairHalfN = 128;
constexpr int kPairStageBytes = (kBM + kPairHalfN) * kBK * 2;
constexpr int kPairGroupT = 8;  // token tiles per group of the tile order (their X tiles stay in L2)
// seven stages (224 KB) where the epilogue stages nothing in shared memory, six beside SWIGLU's 4 KB rows
__host__ __device__ constexpr int pair_stages(int epi) { return epi == TC_SWIGLU ? 6 : 7; }
__host__ __device__ constexpr int pair_smem(int epi) {
    return pair_stages(epi) * kPairStageBytes + 1024 + (epi == TC_SWIGLU ? 4096 : 0);
}

__device__ __forceinline__ TileCoord pair_tile_coord(int tile, int nf, int nt, int gt) {
    TileCoord c;
    const int per_group = nf * gt;
    const int g = tile / per_group, r = tile % per_group;
    const int t_in = min(gt, nt - g * gt);
    c.t0 = g * gt + r % t_in;
    c.f0 = (r / t_in) * kPairBM;
    c.ks = 0;
    c.kb0 = 0;
    c.kb1 = 0;
    return c;
}

template <int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
    qw_tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                           const TcArgs a) {
    constexpr int S = pair_stages(EPI);
    constexpr int A_BYTES = kBM * kBK * 2, B_BYTES = kPairHalfN * kBK * 2;
    constexpr uint32_t TMEM_COLS = 2 * kPairBN;
    constexpr uint32_t IDESC = tc_idesc_f16(kPairBM, kPairBN);
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[S], empty_bar[S], tfull_bar[2], tempty_bar[2], done_bar;
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;

    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *sA = smem;
    uint8_t *sB = smem + S * A_BYTES;
    uint8_t *sStage = smem + S * (A_BYTES + B_BYTES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    volatile int *abort_flag = &abort_sh;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&tfull_bar[i], 1);
            mbar_init(&tempty_bar[i], 8);
        }
        mbar_init(&done_bar, 1);
        abort_sh = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmW) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmX) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA arrival
    tc_fence_after();
    const uint32_t tmem = tmem_base_sh;
    griddep_launch_dependents();

    const int nf = (a.M + kPairBM - 1) / kPairBM, nt = (a.T + kPairBN - 1) / kPairBN;
    const int nkb = (a.K + kBK - 1) / kBK;
    const int total = nf * nt;
    const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer (both CTAs) ----------------
            const uint32_t full0 = cluster_map(smem_u32(&full_bar[0]), 0);
            int s = 0;
            uint32_t ph = 0, issued = 0, last_ph = 0;
            bool ok = true, waited = false;
            int npend = 0, pend_kb[S], pend_t[S];
            auto flush = [&]() {
                griddep_wait();
                waited = true;
                for (int i = 0; i < npend; i++)
                    tma_load_2d_pair(sB + i * B_BYTES, &tmX, full0 + 8u * i, pend_kb[i] * kBK, pend_t[i]);
            };
            for (int tile = cid; tile < total && ok; tile += ncl) {
                const TileCoord c = pair_tile_coord(tile, nf, nt, a.group_t);
                const int wrow = c.f0 + (int)rank * kBM, trow = c.t0 * kPairBN + (int)rank * kPairHalfN;
                for (int kb = 0; kb < nkb; kb++) {
                    if (!mbar_wait(&empty_bar[s], ph ^ 1u, abort_flag, a.err)) { ok = false; break; }
                    if (leader) mbar_arrive_expect_tx(&full_bar[s], 2 * (A_BYTES + B_BYTES));
                    tma_load_2d_pair(sA + s * A_BYTES, &tmW, full0 + 8u * s, kb * kBK, wrow);
                    if (waited) {
                        tma_load_2d_pair(sB + s * B_BYTES, &tmX, full0 + 8u * s, kb * kBK, trow);
                    } else {
                        pend_kb[npend] = kb;
                        pend_t[npend] = trow;
                        if (++npend == S) flush();
                    }
                    issued |= 1u << s;
                    last_ph = (last_ph & ~(1u << s)) | (ph << s);
                    if (++s == S) { s = 0; ph ^= 1u; }
                }
            }
            if (!waited) flush();
            if (!ok && leader) {
                for (int i = 0; i < S; i++)
                    if (issued >> i & 1u) {
                        const uint32_t addr = smem_u32(&full_bar[i]);
                        const uint64_t t0 = gtime_ns();
                        while (!mbar_try(addr, (last_ph >> i) & 1u) && gtime_ns() - t0 < kTcuWaitCycles) {
                        }
                    }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ---------------- MMA issuer (even CTA) ----------------
            int s = 0, it = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int tile = cid; tile < total && ok; tile += ncl, it++) {
                const int acc = it & 1;
                const uint32_t aph = (uint32_t)(it >> 1) & 1u;
                if (!mbar_wait(&tempty_bar[acc], aph ^ 1u, abort_flag, a.err)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(acc * kPairBN);
                for (int kb = 0; kb < nkb; kb++) {
                    if (!mbar_wait(&full_bar[s], ph, abort_flag, a.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t ad = sw128_desc(smem_u32(sA + s * A_BYTES));
                    const uint64_t bd = sw128_desc(smem_u32(sB + s * B_BYTES));
#pragma unroll
                    for (int k = 0; k < kBK / 16; k++)
                        tc_mma_pair(d, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), IDESC, (kb > 0 || k > 0) ? 1u : 0u);
                    tc_commit_pair(&empty_bar[s]);
                    if (++s == S) { s = 0; ph ^= 1u; }
                }
                if (ok) tc_commit_pair(&tfull_bar[acc]);
            }
            tc_commit_pair(&done_bar);
        }
    } else {
        // ---------------- epilogue (warps 2..5 of both CTAs) ----------------
        griddep_wait();
        const uint32_t tempty0 = cluster_map(smem_u32(&tempty_bar[0]), 0);
        const int q = warp & 3;
        int it = 0;
        for (int tile = cid; tile < total; tile += ncl, it++) {
            TileCoord c = pair_tile_coord(tile, nf, nt, a.group_t);
            c.f0 += (int)rank * kBM;  // this CTA's 128 features
            const int acc = it & 1;
            const uint32_t aph = (uint32_t)(it >> 1) & 1u;
            if (!mbar_wait(&tfull_bar[acc], aph, abort_flag, a.err)) break;
            tc_fence_after();
            const int f = c.f0 + q * 32 + lane;
            const int tbase = c.t0 * kPairBN;
            const int ncols = min(kPairBN, a.T - tbase);
            for (int cc = 0; cc < ncols; cc += 32) {
                uint32_t r[32];
                tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * kPairBN + cc), r);
                const int nj = min(32, ncols - cc);
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
                tc_emit<EPI>(a, v, c, f, q, lane, tbase + cc, nj, 0, sStage);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty0 + 8u * (uint32_t)acc);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1 && lane == 0) {
        // every MMA of the pair has completed (they read both CTAs' shared memory and write both TMEMs)
        const uint32_t addr = smem_u32(&done_bar);
        const uint64_t t0 = gtime_ns();
        while (!mbar_try(addr, 0) && gtime_ns() - t0 < kTcuWaitCycles) {
        }
    }
    __syncthreads();
    cluster_sync_all();  // no CTA leaves while its peer may still signal its barriers
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
// bf16 (rows, cols) row-major, box of box_rows x 64 columns, 128-byte swizzle, zero fill
cudaError_t make_map(CUtensorMap *m, const void *base, int rows, int cols, int box_rows) {
    return tma_map_bf16_sw128(m, base, rows, cols, cols, box_rows);
}

template <int BN, int EPI>
cudaError_t launch_bn(const CUtensorMap &mw, const CUtensorMap &mx, const TcArgs &a, int num_sms, cudaStream_t st) {
    auto kfn = qw_tc_gemm_kernel<BN, EPI>;
    const int nf = (a.M + kBM - 1) / kBM, nt = (a.T + BN - 1) / BN;
    const int total = nf * nt * a.ksplit;
    const int grid = total < num_sms ? total : num_sms;
    return launch_pdl(kfn, dim3(grid), dim3(kTcThreads), tc_smem_bytes(BN), st, mw, mx, a);
}

template <int EPI>
cudaError_t launch_pair(const CUtensorMap &mw, const CUtensorMap &mx, const TcArgs &a_in, int num_sms, cudaStream_t st) {
    TcArgs a = a_in;
    static const int gt_env = [] {
        const char *e = getenv("QW_TC_GROUP");
        return e ? atoi(e) : 0;
    }();
    a.group_t = gt_env > 0 ? gt_env : kPairGroupT;
    const int total = ((a.M + kPairBM - 1) / kPairBM) * ((a.T + kPairBN - 1) / kPairBN);
    const int ncl = total < num_sms / 2 ? total : num_sms / 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * ncl);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = pair_smem(EPI);
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, qw_tc_gemm_pair_kernel<EPI>, mw, mx, a);
}

template <int EPI>
cudaError_t launch_epi(const CUtensorMap &mw, const CUtensorMap &mx, const TcArgs &a, int bn, int num_sms,
                       cudaStream_t st) {
    switch (bn) {
        case 64: return launch_bn<64, EPI>(mw, mx, a, num_sms, st);
        case 128: return launch_bn<128, EPI>(mw, mx, a, num_sms, st);
        case 256: return launch_bn<256, EPI>(mw, mx, a, num_sms, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

cudaError_t tma_map_bf16_sw128(CUtensorMap *m, const void *base, long long rows, int cols, int ld, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld % 8) || cols > ld || box_rows < 1 || box_rows > 256)
        return cudaErrorMisalignedAddress;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int EPI>
static cudaError_t prepare_epi() {
    const void *fns[] = {(const void *)qw_tc_gemm_kernel<64, EPI>, (const void *)qw_tc_gemm_kernel<128, EPI>,
                         (const void *)qw_tc_gemm_kernel<256, EPI>};
    const int bns[] = {64, 128, 256};
    for (int i = 0; i < 3; i++) {
        cudaError_t e = cudaFuncSetAttribute(fns[i], cudaFuncAttributeMaxDynamicSharedMemorySize, tc_smem_bytes(bns[i]));
        if (e != cudaSuccess) return e;
    }
    if (EPI == TC_ARGMAX) return cudaSuccess;
    return cudaFuncSetAttribute((const void *)qw_tc_gemm_pair_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                pair_smem(EPI));
}

cudaError_t tc_prepare() {
    cudaError_t e = prepare_epi<TC_STORE>();
    if (e == cudaSuccess) e = prepare_epi<TC_RESID>();
    if (e == cudaSuccess) e = prepare_epi<TC_SWIGLU>();
    if (e == cudaSuccess) e = prepare_epi<TC_ARGMAX>();
    return e;
}

// QW_TC_PAIR=0 keeps prefill shapes on the one-CTA kernel (A/B measurements)
bool tc_pair_enabled() {
    static const bool on = [] {
        const char *e = getenv("QW_TC_PAIR");
        return !(e && e[0] == '0');
    }();
    return on;
}

int tc_pick_bn(int T) { return T <= 64 ? 64 : (T <= 128 ? 128 : 256); }

// K ranges per output tile for a skinny (decode) problem.  A CTA's time is about (work units it runs) x (k-blocks
// per unit + the unit's epilogue, ~2 k-blocks of time for its atomic accumulation), so the split minimising
// ceil(tiles x ks / SMs) x (ceil(k-blocks / ks) + 2) is taken: e.g. 32 tiles x 64 k-blocks -> 4 (one unit per
// CTA), not 5 (160 units: a second unit on 12 CTAs doubles the time).
int tc_pick_ksplit(int M, int T, int K, int bn, int num_sms) {
    const int tiles = ((M + kBM - 1) / kBM) * ((T + bn - 1) / bn);
    const int nkb = (K + kBK - 1) / kBK;
    if (tiles >= 2 * num_sms || (bn > 64 && tiles >= num_sms / 2)) return 1;  // prefill shapes: no split
    int best_ks = 1;
    long long best = -1;
    for (int ks = 1; ks <= (nkb / 2 > 1 ? nkb / 2 : 1); ks++) {  // at least two k-blocks per split
        const long long waves = ((long long)tiles * ks + num_sms - 1) / num_sms;
        const long long cost = waves * ((nkb + ks - 1) / ks + 2);
        if (best < 0 || cost < best) { best = cost; best_ks = ks; }
    }
    return best_ks;
}

cudaError_t tc_gemm_launch(const void *W, const void *X, const TcArgs &a, int epi, int bn, int num_sms,
                           cudaStream_t st) {
    if (a.M < 1 || a.T < 1 || a.K < 8 || a.K % 8 || a.ksplit < 1) return cudaErrorInvalidValue;
    if (a.ksplit > (a.K + kBK - 1) / kBK) return cudaErrorInvalidValue;
    if (epi == TC_SWIGLU && (a.ksplit != 1 || a.M % 32)) return cudaErrorInvalidValue;
    if (epi == TC_ARGMAX && (a.ksplit != 1 || !a.cand_val || !a.cand_idx || a.ncand < (a.M + kBM - 1) / kBM * 4))
        return cudaErrorInvalidValue;
    if (epi == TC_RESID && a.ksplit > 1 && a.out != (const void *)a.resid) return cudaErrorInvalidValue;
    if (bn == 0) bn = tc_pick_bn(a.T);
    CUtensorMap mw, mx;
    if (bn == 256 && a.ksplit == 1 && epi != TC_ARGMAX && tc_pair_enabled() &&
        ((a.M + kPairBM - 1) / kPairBM) * ((a.T + kPairBN - 1) / kPairBN) >= num_sms / 2) {
        // prefill shapes: the CTA-pair kernel (each CTA maps 128-row boxes of W and of X)
        cudaError_t e = make_map(&mw, W, a.M, a.K, kBM);
        if (e == cudaSuccess) e = make_map(&mx, X, a.T, a.K, kPairHalfN);
        if (e != cudaSuccess) return e;
        switch (epi) {
            case TC_STORE: return launch_pair<TC_STORE>(mw, mx, a, num_sms, st);
            case TC_RESID: return launch_pair<TC_RESID>(mw, mx, a, num_sms, st);
            case TC_SWIGLU: return launch_pair<TC_SWIGLU>(mw, mx, a, num_sms, st);
        }
        return cudaErrorInvalidValue;
    }
    cudaError_t e = make_map(&mw, W, a.M, a.K, kBM);
    if (e != cudaSuccess) return e;
    e = make_map(&mx, X, a.T, a.K, bn);
    if (e != cudaSuccess) return e;
    switch (epi) {
        case TC_STORE: return launch_epi<TC_STORE>(mw, mx, a, bn, num_sms, st);
        case TC_RESID: return launch_epi<TC_RESID>(mw, mx, a, bn, num_sms, st);
        case TC_SWIGLU: return launch_epi<TC_SWIGLU>(mw, mx, a, bn, num_sms, st);
        case TC_ARGMAX: return launch_epi<TC_ARGMAX>(mw, mx, a, bn, num_sms, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace qw

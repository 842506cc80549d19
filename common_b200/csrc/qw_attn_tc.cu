// qw_attn_tc.cu -- causal GQA prefill attention on the 5th-generation tensor cores (head_dim 128).
//
// Semantics: scores q . k / sqrt(d) (AttentionFeatures.java:531-559), the causal mask (:906-917; future keys
// contribute nothing), log-stable softmax (ActivationFeatures.java:136-142) and the value sum
// (AttentionFeatures.java:572-616) over the paged bf16 KV cache, fp32 accumulation, online-softmax tiling.
//
// One CTA = two query tiles of 128 rows, each 128 / G consecutive positions of each of the G query heads of
// one KV head (G = heads per KV head), so every K / V block it loads serves both tiles and all G heads.
// Blocks of 128 keys.
//   warp 0      TMA producer: the two Q tiles once (boxes of 128 / G rows x 2 column halves), then for every
//               key block its K and V tiles from the paged cache (boxes of min(page, 128) rows, two 64-column
//               halves, 128-byte swizzle) into 2-stage rings; no multicast;
//   warp 1      allocates all 512 TMEM columns (S_0, S_1, O_0, O_1); one lane issues, for every key block,
//               S_0 = Q_0 K^T, S_1 = Q_1 K^T (M 128, N 128, 8 x K=16), then O_t += P_t V as soon as tile t's
//               softmax has written P_t: while warps 2..5 work on tile 0 the tensor cores run tile 1 and back
//               (ping-pong).  P_t is read from TMEM (packed bf16 pairs over the first 64 columns of S_t); V is
//               the MN-major shared-memory operand, exactly its cache layout;
//   warps 2..9  softmax of tile (warp - 2) / 4, one query row per thread: S row from TMEM, mask, scale into
//               log2 units, online softmax with a lazily updated maximum (O and the row sum are rescaled only
//               when the maximum grows by more than 2^8; the values between stay below 2^8), P into TMEM;
//               finally O / l as bf16 rows.
// Every mbarrier wait is bounded; on expiry the CTA records the timeout, lets its copies and MMAs land, frees
// its TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>

#include "qw_internal.cuh"
#include "qw_kernels.h"
#include "qw_tc.h"
#include "qw_tc_util.cuh"

namespace qw {

namespace {

constexpr int kAtThreads = 320;
constexpr int kAtRows = 128, kAtKeys = 128, kAtD = 128;
constexpr int kAtHalf = kAtRows * 64 * 2;  // 16 KiB: 128 rows x 64 bf16 columns
constexpr int kAtTile = 2 * kAtHalf;       // 32 KiB: a 128 x 128 bf16 operand
constexpr int kAtSmem = 6 * kAtTile + 1024;  // Q[2] | K[2] | V[2], 1 KiB alignment slack
constexpr uint32_t kAtTmemCols = 512;
constexpr float kAtRescale = 8.f;

// K-major or MN-major 128-byte-swizzled operand descriptor; lbo / sbo in bytes
__device__ __forceinline__ uint64_t sw128_desc2(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

__device__ __forceinline__ void tmem_ld32_nw(uint32_t taddr, float *v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float *v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
        "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
        "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
        "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

struct AtParams {
    int L, p0, G, rph, ntile, Hkv, ps, lg, max_pages;
    const int *page_table, *seq_slots;
    float sl2;  // scale * log2(e)
    __nv_bfloat16 *out;
    int ld_out;
    int *err;
};
// tcgen05.mma with the A operand (P) in tensor memory: two bf16 per 32-bit column along K
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                          uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t *r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__global__ void __launch_bounds__(kAtThreads, 1)
    qw_flash_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                               const __grid_constant__ CUtensorMap tmV, const AtParams a) {
    extern __shared__ uint8_t at_smem_raw[];
    __shared__ __align__(8) uint64_t q_full, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2], p_full[2],
        o_full[2], done_bar;
    __shared__ uint32_t tmem_sh;
    __shared__ int abort_sh;
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(at_smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *sQ = sm, *sK = sm + 2 * kAtTile, *sV = sm + 4 * kAtTile;  // Q[2] | K[2] | V[2]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    volatile int *abort_flag = &abort_sh;

    const int qt = a.ntile - 1 - (int)blockIdx.x;  // the longest (latest) tiles first
    const int kvh = blockIdx.y, b = blockIdx.z;
    const int q0 = qt * 2 * a.rph;                           // first position (within the chunk) of query tile 0
    const int plast = a.p0 + min(a.L, q0 + 2 * a.rph) - 1;  // the CTA's last position
    const int nblk = plast / kAtKeys + 1;

    if (threadIdx.x == 0) {
        mbar_init(&q_full, 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 4);
            mbar_init(&o_full[i], 1);
        }
        mbar_init(&done_bar, 1);
        abort_sh = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmQ) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmK) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmV) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_sh)),
                     "r"(kAtTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_sh;
    griddep_launch_dependents();
    griddep_wait();  // q and the cache rows of this chunk come from the previous kernel

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            const int *ptab = a.page_table + (size_t)a.seq_slots[b] * a.max_pages;
            const int br = min(a.ps, kAtKeys), nbox = kAtKeys / br;
            mbar_arrive_expect_tx(&q_full, 2 * kAtTile);
            for (int t = 0; t < 2; t++)
                for (int g = 0; g < a.G; g++)
                    for (int c = 0; c < 2; c++)
                        tma_load_2d(sQ + t * kAtTile + c * kAtHalf + g * a.rph * 128, &tmQ, &q_full,
                                    (kvh * a.G + g) * kAtD + c * 64, b * a.L + q0 + t * a.rph);
            uint32_t issued_k = 0, issued_v = 0, ph_k = 0, ph_v = 0;
            bool ok = true;
            for (int j = 0; j < nblk && ok; j++) {
                const int s = j & 1;
                const uint32_t ph = (uint32_t)(j >> 1) & 1u;
                for (int which = 0; which < 2 && ok; which++) {
                    uint64_t *emp = which ? &v_empty[s] : &k_empty[s];
                    uint64_t *ful = which ? &v_full[s] : &k_full[s];
                    if (!mbar_wait(emp, ph ^ 1u, abort_flag, a.err)) { ok = false; break; }
                    mbar_arrive_expect_tx(ful, kAtTile);
                    uint8_t *dst = (which ? sV : sK) + s * kAtTile;
                    for (int i = 0; i < nbox; i++) {
                        const int t = j * kAtKeys + i * br;
                        // boxes past the CTA's last position read the zero fill (finite values under P = 0)
                        const int y = t <= plast ? (ptab[t >> a.lg] * a.Hkv + kvh) * a.ps + (t & (a.ps - 1)) : -br;
                        for (int c = 0; c < 2; c++)
                            tma_load_2d(dst + c * kAtHalf + i * br * 128, which ? &tmV : &tmK, ful, c * 64, y);
                    }
                    if (which) { issued_v |= 1u << s; ph_v = (ph_v & ~(1u << s)) | (ph << s); }
                    else { issued_k |= 1u << s; ph_k = (ph_k & ~(1u << s)) | (ph << s); }
                }
            }
            if (!ok) {  // let every issued copy land before the shared memory goes away
                const uint64_t t0 = gtime_ns();
                while (!mbar_try(smem_u32(&q_full), 0) && gtime_ns() - t0 < kTcuWaitCycles) {
                }
                for (int s = 0; s < 2; s++) {
                    if (issued_k >> s & 1u)
                        while (!mbar_try(smem_u32(&k_full[s]), (ph_k >> s) & 1u) && gtime_ns() - t0 < kTcuWaitCycles) {
                        }
                    if (issued_v >> s & 1u)
                        while (!mbar_try(smem_u32(&v_full[s]), (ph_v >> s) & 1u) && gtime_ns() - t0 < kTcuWaitCycles) {
                        }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer: tiles 0 and 1 alternate, so that one tile's softmax runs while the
            // tensor cores work on the other ----------------
            constexpr uint32_t IDS = tc_idesc_f16(kAtRows, kAtKeys, 0);  // S = Q K^T: both K-major
            constexpr uint32_t IDP = tc_idesc_f16(kAtRows, kAtD, 1);     // O += P V: P in TMEM, V MN-major
            bool ok = mbar_wait(&q_full, 0, abort_flag, a.err);
            // S_t(j) = Q_t K_j^T into TMEM columns [128 t, 128 t + 128); the MMAs of a thread run in issue order,
            // so S_t(j) overwrites P_t(j - 1) only after PV_t(j - 1) has read it
            auto issue_s = [&](int t, int j) -> bool {
                const int s = j & 1;
                if (t == 0 && !mbar_wait(&k_full[s], (uint32_t)(j >> 1) & 1u, abort_flag, a.err)) return false;
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < kAtD / 16; kk++) {
                    const uint32_t off = (uint32_t)((kk >> 2) * kAtHalf + (kk & 3) * 32);
                    tc_mma(tmem + (uint32_t)(t * kAtKeys), sw128_desc2(smem_u32(sQ + t * kAtTile) + off, 16, 1024),
                           sw128_desc2(smem_u32(sK + s * kAtTile) + off, 16, 1024), IDS, kk > 0 ? 1u : 0u);
                }
                tc_commit(&s_full[t]);  // also covers PV_t(j - 1): O_t is safe to rescale
                if (t == 1) tc_commit(&k_empty[s]);
                return true;
            };
            // O_t += P_t(j) V_j, P_t(j) read from TMEM columns [128 t, 128 t + 64) as packed bf16 pairs
            auto issue_pv = [&](int t, int j) -> bool {
                const int s = j & 1;
                if (!mbar_wait(&p_full[t], (uint32_t)j & 1u, abort_flag, a.err)) return false;
                if (t == 0 && !mbar_wait(&v_full[s], (uint32_t)(j >> 1) & 1u, abort_flag, a.err)) return false;
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < kAtKeys / 16; kk++)
                    tc_mma_ts(tmem + 256u + (uint32_t)(t * kAtD), tmem + (uint32_t)(t * kAtKeys + kk * 8),
                              sw128_desc2(smem_u32(sV + s * kAtTile) + (uint32_t)(kk * 2048), kAtHalf, 1024), IDP,
                              (j > 0 || kk > 0) ? 1u : 0u);
                if (t == 1) tc_commit(&v_empty[s]);
                if (j == nblk - 1) tc_commit(&o_full[t]);
                return true;
            };
            if (ok) ok = issue_s(0, 0) && issue_s(1, 0);
            for (int j = 0; j < nblk && ok; j++) {
                ok = issue_pv(0, j);
                if (ok && j + 1 < nblk) ok = issue_s(0, j + 1);
                if (ok) ok = issue_pv(1, j);
                if (ok && j + 1 < nblk) ok = issue_s(1, j + 1);
            }
            // every MMA of this CTA has completed before the TMEM is freed
            tc_commit(&done_bar);
            const uint64_t t0 = gtime_ns();
            while (!mbar_try(smem_u32(&done_bar), 0) && gtime_ns() - t0 < kTcuWaitCycles) {
            }
        }
    } else {
        // ---------------- softmax + epilogue: warps 2..5 query tile 0, warps 6..9 tile 1, one row per thread ----
        const int t = (warp - 2) >> 2;  // query tile
        const int qq = warp & 3;        // TMEM lane quarter of this warp
        const int row = qq * 32 + lane;
        const int g = row / a.rph, pl = t * a.rph + row % a.rph;  // head, position offset within the CTA
        const bool valid = q0 + pl < a.L;
        const int pos = valid ? a.p0 + q0 + pl : plast;
        const uint32_t trow = tmem + ((uint32_t)(qq * 32) << 16);
        const uint32_t ts = trow + (uint32_t)(t * kAtKeys), to = trow + 256u + (uint32_t)(t * kAtD);
        float m_use = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nblk && ok; j++) {
            if (!mbar_wait(&s_full[t], (uint32_t)j & 1u, abort_flag, a.err)) { ok = false; break; }
            tc_fence_after();
            float v[kAtKeys];
#pragma unroll
            for (int c = 0; c < 4; c++) tmem_ld32_nw(ts + (uint32_t)(c * 32), v + c * 32);
            tmem_wait_ld();
            const int kbase = j * kAtKeys;
            // maximum of the raw scores (the scale is positive), 4 independent chains
            float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
            if (kbase + kAtKeys - 1 > pos) {
#pragma unroll
                for (int e = 0; e < kAtKeys; e++) {
                    if (kbase + e > pos) v[e] = -INFINITY;
                    m4[e & 3] = fmaxf(m4[e & 3], v[e]);
                }
            } else {
#pragma unroll
                for (int e = 0; e < kAtKeys; e++) m4[e & 3] = fmaxf(m4[e & 3], v[e]);
            }
            const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * a.sl2;
            float alpha = 1.f;
            bool need = false;
            if (j == 0) {
                m_use = mx;  // key 0 <= pos: finite
            } else if (mx > m_use + kAtRescale) {
                alpha = ex2(m_use - mx);
                m_use = mx;
                need = true;
            }
            // p = 2^(s * scale * log2 e - m): one FMA and one ex2 per score; P_t(j) goes to TMEM as packed bf16
            // pairs over the first 64 columns of S_t(j), 16 columns (32 scores) at a time
            float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < 4; c++) {
                uint32_t pk[16];
#pragma unroll
                for (int e = 0; e < 32; e += 2) {
                    const float p0 = ex2(fmaf(v[c * 32 + e], a.sl2, -m_use)), p1 = ex2(fmaf(v[c * 32 + e + 1], a.sl2, -m_use));
                    s4[(e >> 1) & 3] += p0 + p1;
                    pk[e / 2] = pack2(p0, p1);
                }
                tmem_st16u(ts + (uint32_t)(c * 16), pk);
            }
            const float sum = (s4[0] + s4[1]) + (s4[2] + s4[3]);
            l = l * alpha + sum;
            // O_t: PV_t(j - 1) has completed (s_full of this block was committed after it)
            if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    float o[32];
                    tmem_ld32_nw(to + (uint32_t)(c * 32), o);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; e++) o[e] *= alpha;
                    tmem_st32(to + (uint32_t)(c * 32), o);
                }
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[t]);
        }
        if (ok && mbar_wait(&o_full[t], 0, abort_flag, a.err)) {
            tc_fence_after();
            const float inv = l > 0.f ? 1.0f / l : 0.f;
            __nv_bfloat16 *orow = a.out + (size_t)(b * a.L + q0 + pl) * a.ld_out + (size_t)(kvh * a.G + g) * kAtD;
#pragma unroll
            for (int c = 0; c < 4; c++) {
                float o[32];
                tmem_ld32_nw(to + (uint32_t)(c * 32), o);
                tmem_wait_ld();
                if (valid) {
#pragma unroll
                    for (int e = 0; e < 32; e += 8) {
                        uint4 w;
                        w.x = pack2(o[e] * inv, o[e + 1] * inv);
                        w.y = pack2(o[e + 2] * inv, o[e + 3] * inv);
                        w.z = pack2(o[e + 4] * inv, o[e + 5] * inv);
                        w.w = pack2(o[e + 6] * inv, o[e + 7] * inv);
                        *reinterpret_cast<uint4 *>(orow + c * 32 + e) = w;
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kAtTmemCols) : "memory");
    }
}

}  // namespace

cudaError_t flash_prefill_tc_prepare() {
    return cudaFuncSetAttribute(qw_flash_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAtSmem);
}

cudaError_t flash_prefill_tc_launch(const FlashArgs &fa, int nseq, cudaStream_t st) {
    if (fa.d != kAtD) return cudaErrorInvalidValue;
    const int G = fa.H / fa.Hkv;
    if (G < 1 || G > 8 || (G & (G - 1)) || fa.page_size < 16 || fa.num_pages < 1) return cudaErrorInvalidValue;
    AtParams a{};
    a.L = fa.L; a.p0 = fa.p0; a.G = G; a.rph = kAtRows / G; a.ntile = (fa.L + 2 * a.rph - 1) / (2 * a.rph);
    a.Hkv = fa.Hkv; a.ps = fa.page_size; a.lg = fa.log2_page; a.max_pages = fa.max_pages;
    a.page_table = fa.page_table; a.seq_slots = fa.seq_slots;
    a.sl2 = fa.scale * 1.4426950408889634f;
    a.out = fa.out; a.ld_out = fa.ld_out; a.err = fa.err;
    CUtensorMap mq, mk, mv;
    cudaError_t e = tma_map_bf16_sw128(&mq, fa.q, (long long)nseq * fa.L, fa.H * kAtD, fa.ld_q, a.rph);
    if (e != cudaSuccess) return e;
    const long long crow = (long long)fa.num_pages * fa.Hkv * fa.page_size;
    const int br = fa.page_size < kAtKeys ? fa.page_size : kAtKeys;
    e = tma_map_bf16_sw128(&mk, fa.kcache, crow, kAtD, kAtD, br);
    if (e != cudaSuccess) return e;
    e = tma_map_bf16_sw128(&mv, fa.vcache, crow, kAtD, kAtD, br);
    if (e != cudaSuccess) return e;
    return launch_pdl(qw_flash_prefill_tc_kernel, dim3(a.ntile, fa.Hkv, nseq), dim3(kAtThreads), kAtSmem, st, mq, mk,
                      mv, a);
}

}  // namespace qw

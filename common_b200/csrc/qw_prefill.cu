// qw_prefill.cu -- kernels around the tensor-core projections of prefill and batched decode.
//
//   norm_rows     residual stream update (embedding gather for layer 0, plus an all-reduced
//                 partial under tensor parallelism) and rmsnorm (NormalizationLayerFeatures.java:
//                 587-603) of every token row into the bf16 operand of the next GEMM;
//   qkv_post      per token: QK-norm (whole-vector as the reference, AttentionFeatures.java:840-845,
//                 886-891, or per head), split-half RoPE (RotationFeatures.java:124-170, 189-208),
//                 the paged KV-cache write (AttentionFeatures.java:823-877) and the bf16 query row;
//   flash_prefill causal GQA attention of a chunk of prompt positions over the paged cache
//                 (scores AttentionFeatures.java:531-559, mask :906-917, log-stable softmax
//                 ActivationFeatures.java:136-142, PV AttentionFeatures.java:572-616) as the
//                 online-softmax tiling on bf16 mma.sync tensor-core tiles, fp32 accumulation;
//   rows_argmax   first index of the maximum of each logits row (AggregationFeatures.java:111-121).
#include "qw_internal.cuh"
#include "qw_kernels.h"
#include "qw_ar.h"
#include "qw_tc.h"
#include "qw_tc_util.cuh"
#include <float.h>
#include <limits.h>

namespace qw {

// ------------------------------------------------------------------------------------------
// norm_rows: one CTA per token row
// ------------------------------------------------------------------------------------------
constexpr int kNormThreads = 256;  // 8 rows per SM in flight (16 KB of shared memory each)
constexpr size_t kPrepSmem = 160 * 1024;  // dynamic shared memory the row kernels are opted in to

__global__ void __launch_bounds__(kNormThreads) qw_norm_rows_kernel(NormRowsArgs a) {
    griddep_launch_dependents();  // programmatic launch: the next kernel may start its prologue
    griddep_wait();               // the previous kernel's results
    extern __shared__ __align__(16) float xrow[];
    __shared__ float red[kNormThreads / 32];
    const int r = blockIdx.x, K = a.K, tid = threadIdx.x;
    const __nv_bfloat16 *erow = a.embed ? a.embed + (size_t)a.tokens[r] * K : nullptr;
    float ss = 0.f;
    for (int k = tid * 4; k < K; k += kNormThreads * 4) {
        float4 v;
        if (erow) {
            uint2 u = *reinterpret_cast<const uint2 *>(erow + k);
            v = make_float4(bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y));
        } else {
            v = *reinterpret_cast<const float4 *>(a.x + (size_t)r * a.ld_x + k);
        }
        if (a.part) {
            float4 p = *reinterpret_cast<const float4 *>(a.part + (size_t)r * a.ld_part + k);
            if (a.zero_part) *reinterpret_cast<float4 *>(a.part + (size_t)r * a.ld_part + k) = make_float4(0.f, 0.f, 0.f, 0.f);
            v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
        }
        if (erow || a.part) *reinterpret_cast<float4 *>(a.x + (size_t)r * a.ld_x + k) = v;
        *reinterpret_cast<float4 *>(xrow + k) = v;
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kNormThreads / 32; w++) tot += red[w];
    const float sc = 1.0f / sqrtf(tot / (float)K + a.eps);
    for (int k = tid * 4; k < K; k += kNormThreads * 4) {
        float4 v = *reinterpret_cast<const float4 *>(xrow + k);
        float4 w = *reinterpret_cast<const float4 *>(a.w + k);
        uint2 o;
        o.x = (uint32_t)f2bf_bits(w.x * v.x * sc) | ((uint32_t)f2bf_bits(w.y * v.y * sc) << 16);
        o.y = (uint32_t)f2bf_bits(w.z * v.z * sc) | ((uint32_t)f2bf_bits(w.w * v.w * sc) << 16);
        *reinterpret_cast<uint2 *>(a.out + (size_t)r * a.ld_out + k) = o;
    }
}

cudaError_t norm_rows_launch(const NormRowsArgs &a, int rows, cudaStream_t st) {
    if (rows < 1 || a.K % 4) return cudaErrorInvalidValue;
    size_t smem = sizeof(float) * a.K;
    if (smem > kPrepSmem) return cudaErrorInvalidValue;
    return launch_pdl(qw_norm_rows_kernel, dim3(rows), dim3(kNormThreads), smem, st, a);
}

// ------------------------------------------------------------------------------------------
// qkv_post: one CTA per token row
// ------------------------------------------------------------------------------------------
constexpr int kPostThreads = 256;
constexpr unsigned long long kXwWaitCycles = 4000ull * 1000ull * 1000ull;  // ~2 s at 2 GHz

// 8 consecutive values to the cache type: one 16-byte store (bf16) or two (fp32)
__device__ __forceinline__ void store8(__nv_bfloat16 *p, const float (&v)[8]) {
    uint4 u;
    u.x = (uint32_t)f2bf_bits(v[0]) | ((uint32_t)f2bf_bits(v[1]) << 16);
    u.y = (uint32_t)f2bf_bits(v[2]) | ((uint32_t)f2bf_bits(v[3]) << 16);
    u.z = (uint32_t)f2bf_bits(v[4]) | ((uint32_t)f2bf_bits(v[5]) << 16);
    u.w = (uint32_t)f2bf_bits(v[6]) | ((uint32_t)f2bf_bits(v[7]) << 16);
    *reinterpret_cast<uint4 *>(p) = u;
}
__device__ __forceinline__ void store8(float *p, const float (&v)[8]) {
    reinterpret_cast<float4 *>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4 *>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// One row: QK-norm (AttentionFeatures.java:840-845, 886-891 whole-vector; or per head), split-half RoPE
// (RotationFeatures.java:189-208) of q and k, bf16 queries out, k and v into the paged cache.  The row is
// loaded once (16-byte loads) into shared memory; then one pass in which a thread takes 8 columns of the first
// half of a head together with the matching 8 of its second half (a RoPE pair), or 8 columns of v.
template <typename KT>
__global__ void __launch_bounds__(kPostThreads) qw_qkv_post_kernel(QkvPostArgs a) {
    griddep_launch_dependents();  // programmatic launch: the next kernel may start its prologue
    griddep_wait();               // the previous kernel's results
    extern __shared__ __align__(16) float row[];  // q (Ql) | k (KVl) | v (KVl)
    __shared__ float red[2][kPostThreads / 32];
    __shared__ float s_sc[2];
    __shared__ float s_head[128];  // per-head scales (qk_mode 2)
    const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int d = a.d, Ql = a.H * d, KVl = a.Hkv * d, W = Ql + 2 * KVl;
    const float *src = a.qkv + (size_t)r * a.ld_qkv;
    unsigned xgen = 0;  // thread 0: generation of the sums exchange
    float sq = 0.f, sk = 0.f;
    for (int i = tid * 4; i < W; i += kPostThreads * 4) {
        const float4 v = *reinterpret_cast<const float4 *>(src + i);
        *reinterpret_cast<float4 *>(row + i) = v;
        const float s2 = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        if (i < Ql) sq += s2;
        else if (i < Ql + KVl) sk += s2;
    }
    if (a.zero_qkv) {
        // zeroed again for the next split-K accumulation into this buffer (after all loads of the row)
        __syncthreads();
        for (int i = tid * 4; i < W; i += kPostThreads * 4)
            *reinterpret_cast<float4 *>(a.qkv + (size_t)r * a.ld_qkv + i) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (a.qk_mode == 1) {
        sq = warp_sum(sq);
        sk = warp_sum(sk);
        if (lane == 0) { red[0][warp] = sq; red[1][warp] = sk; }
        __syncthreads();
        if (tid == 0) {
            float tq = 0.f, tk = 0.f;
            for (int w = 0; w < kPostThreads / 32; w++) { tq += red[0][w]; tk += red[1][w]; }
            if (a.qk_ss) { tq = a.qk_ss[2 * r]; tk = a.qk_ss[2 * r + 1]; }
            if (a.xpeers) {
                // every rank's two sums of this row, added in rank order (the same scale on every rank)
                xgen = *reinterpret_cast<volatile unsigned *>(a.gen) + 1u;
                for (int p = 0; p < a.tp; p++) {
                    unsigned long long *dst = a.xpeers[p] + a.xoff + ((size_t)r * a.tp + a.rank) * 2;
                    xw_store(dst, tq, xgen);
                    xw_store(dst + 1, tk, xgen);
                }
                const unsigned long long *in = a.xpeers[a.rank] + a.xoff + (size_t)r * a.tp * 2;
                float sq2 = 0.f, sk2 = 0.f;
                bool ok = true;
                unsigned long long w[8][2];  // every rank's pair loaded at once (tp <= 8), then settled in order
#pragma unroll
                for (int p = 0; p < 8; p++)
                    if (p < a.tp) xw_load2(in + 2 * p, w[p][0], w[p][1]);
#pragma unroll
                for (int p = 0; p < 8; p++)
                    if (p < a.tp && ok) {
                        float vq = 0.f, vk = 0.f;
                        ok = xw_settle(in + 2 * p, w[p][0], xgen, vq, kXwWaitCycles) &&
                             xw_settle(in + 2 * p + 1, w[p][1], xgen, vk, kXwWaitCycles);
                        sq2 += vq;
                        sk2 += vk;
                    }
                if (!ok && a.err) atomicExch(a.err, 6);
                tq = sq2;
                tk = sk2;
            }
            s_sc[0] = 1.0f / sqrtf(tq / (float)a.q_total + 1e-6f);
            s_sc[1] = 1.0f / sqrtf(tk / (float)a.kv_total + 1e-6f);
        }
    } else if (a.qk_mode == 2) {
        __syncthreads();
        for (int hh = warp; hh < a.H + a.Hkv; hh += kPostThreads / 32) {
            const float *v = row + (size_t)hh * d;
            float s2 = 0.f;
            for (int i = lane; i < d; i += 32) s2 += v[i] * v[i];
            s2 = warp_sum(s2);
            if (lane == 0) s_head[hh] = 1.0f / sqrtf(s2 / (float)d + 1e-6f);
        }
    }
    __syncthreads();
    const int pos = a.positions[r];
    const int half = d / 2, hc = half / 8;  // 8-column pieces per half head
    const float2 *fr = a.freq + (size_t)pos * half;
    const int slot = a.slots[r];
    const int page = a.page_table[(size_t)slot * a.max_pages + (pos >> a.log2_page)];
    const size_t cache_row = ((size_t)page * a.Hkv * a.page_size + (pos & (a.page_size - 1))) * d;
    KT *kc = reinterpret_cast<KT *>(a.kcache);
    KT *vc = reinterpret_cast<KT *>(a.vcache);
    const int nrope = (a.H + a.Hkv) * hc, nv = KVl / 8;
    for (int it = tid; it < nrope + nv; it += kPostThreads) {
        if (it < nrope) {
            const int hh = it / hc, f0 = (it % hc) * 8;
            const bool isq = hh < a.H;
            const float *v = row + (size_t)hh * d;
            float x1[8], x2[8];
#pragma unroll
            for (int e = 0; e < 8; e += 4) {
                const float4 u1 = *reinterpret_cast<const float4 *>(v + f0 + e);
                const float4 u2 = *reinterpret_cast<const float4 *>(v + f0 + half + e);
                x1[e] = u1.x; x1[e + 1] = u1.y; x1[e + 2] = u1.z; x1[e + 3] = u1.w;
                x2[e] = u2.x; x2[e + 1] = u2.y; x2[e + 2] = u2.z; x2[e + 3] = u2.w;
            }
            if (a.qk_mode == 1) {
                const float sc = isq ? s_sc[0] : s_sc[1];
                const float *w = isq ? a.qn + (size_t)hh * d : a.kn + (size_t)(hh - a.H) * d;
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    x1[e] = w[f0 + e] * x1[e] * sc;
                    x2[e] = w[f0 + half + e] * x2[e] * sc;
                }
            } else if (a.qk_mode == 2) {
                const float sc = s_head[hh];
                const float *w = isq ? a.qn + (size_t)hh * d : a.kn + (size_t)(hh - a.H) * d;
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    x1[e] = w[f0 + e] * x1[e] * sc;
                    x2[e] = w[f0 + half + e] * x2[e] * sc;
                }
            }
            float y1[8], y2[8];
#pragma unroll
            for (int e = 0; e < 8; e++) {
                const float2 cs = fr[f0 + e];
                y1[e] = x1[e] * cs.x - x2[e] * cs.y;
                y2[e] = x2[e] * cs.x + x1[e] * cs.y;
            }
            if (isq) {
                __nv_bfloat16 *q = a.q_out + (size_t)r * a.ld_q + (size_t)hh * d;
                store8(q + f0, y1);
                store8(q + f0 + half, y2);
            } else {
                KT *k = kc + cache_row + (size_t)(hh - a.H) * a.page_size * d;
                store8(k + f0, y1);
                store8(k + f0 + half, y2);
            }
        } else {
            const int c = (it - nrope) * 8, h = c / d, j = c % d;
            const float *v = row + Ql + KVl + c;
            float x[8];
            const float4 u1 = *reinterpret_cast<const float4 *>(v), u2 = *reinterpret_cast<const float4 *>(v + 4);
            x[0] = u1.x; x[1] = u1.y; x[2] = u1.z; x[3] = u1.w; x[4] = u2.x; x[5] = u2.y; x[6] = u2.z; x[7] = u2.w;
            store8(vc + cache_row + (size_t)h * a.page_size * d + j, x);
        }
    }
    if (a.xpeers && a.qk_mode == 1) {
        // the last CTA advances the exchange generation (every CTA has read it)
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            if (atomicAdd(a.done, 1u) == gridDim.x - 1) {
                *a.done = 0u;
                *a.gen = xgen;
            }
        }
    }
}

cudaError_t qkv_post_launch(const QkvPostArgs &a, int rows, bool kv_bf16, cudaStream_t st) {
    size_t smem = sizeof(float) * (size_t)(a.H + 2 * a.Hkv) * a.d;
    if (a.d % 16 || a.H + a.Hkv > 128 || a.ld_qkv % 4 || a.ld_q % 8) return cudaErrorInvalidValue;
    auto k16 = qw_qkv_post_kernel<__nv_bfloat16>;
    auto k32 = qw_qkv_post_kernel<float>;
    if (smem > kPrepSmem) return cudaErrorInvalidValue;
    return kv_bf16 ? launch_pdl(k16, dim3(rows), dim3(kPostThreads), smem, st, a)
                   : launch_pdl(k32, dim3(rows), dim3(kPostThreads), smem, st, a);
}

// ------------------------------------------------------------------------------------------
// flash_prefill: grid (query tiles of 64, query heads, sequences), 4 warps x 16 query rows
// ------------------------------------------------------------------------------------------
constexpr int kFaRows = 64, kFaKeys = 64, kFaWarps = 4;
constexpr int kFaMaxSplit = 64;

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    return (uint32_t)f2bf_bits(lo) | ((uint32_t)f2bf_bits(hi) << 16);
}

// byte offset of (row, 16-byte chunk) in a [rows][D] bf16 tile, chunks XOR-swizzled by row
template <int D>
__device__ __forceinline__ uint32_t fa_off(int row, int chunk) {
    return (uint32_t)(row * D * 2 + ((chunk ^ (row & 7)) << 4));
}

template <int D>
__global__ void __launch_bounds__(kFaWarps * 32) qw_flash_prefill_kernel(FlashArgs a) {
    griddep_launch_dependents();  // programmatic launch: the next kernel may start its prologue
    griddep_wait();               // the previous kernel's results
    constexpr int CH = D / 8;  // 16-byte chunks per row
    extern __shared__ __align__(128) uint8_t fsm[];
    uint8_t *sK = fsm;                      // [2][64][D]
    uint8_t *sV = fsm + 2 * kFaKeys * D * 2;  // [2][64][D]
    const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const int G = a.H / a.Hkv, kvh = h / G;
    const int q0 = qt * kFaRows;  // first query row of the tile within this sequence's chunk
    if (q0 >= a.L) return;
    const int slot = a.seq_slots[b];
    const int *ptab = a.page_table + (size_t)slot * a.max_pages;
    const int qpos0 = a.p0 + q0;                              // position of the tile's first query
    const int qlast = a.p0 + min(a.L, q0 + kFaRows) - 1;      // position of its last query
    const int nkt = qlast / kFaKeys + 1;                      // key tiles covering [0, qlast]
    const __nv_bfloat16 *kc = reinterpret_cast<const __nv_bfloat16 *>(a.kcache);
    const __nv_bfloat16 *vc = reinterpret_cast<const __nv_bfloat16 *>(a.vcache);

    auto load_tile = [&](int kt, int buf) {
        const uint32_t bk = smem_addr(sK + buf * kFaKeys * D * 2), bv = smem_addr(sV + buf * kFaKeys * D * 2);
        for (int i = tid; i < kFaKeys * CH; i += kFaWarps * 32) {
            const int r = i / CH, c = i % CH;
            const int pos = kt * kFaKeys + r;
            const bool ok = pos <= qlast;
            const int page = ok ? ptab[pos >> a.log2_page] : 0;
            const size_t off = (((size_t)page * a.Hkv + kvh) * a.page_size + (pos & (a.page_size - 1))) * D + c * 8;
            cp_async16(bk + fa_off<D>(r, c), ok ? kc + off : kc, ok ? 16 : 0);
            cp_async16(bv + fa_off<D>(r, c), ok ? vc + off : vc, ok ? 16 : 0);
        }
        cp_async_commit();
    };
    load_tile(0, 0);

    // this warp's 16 query rows as A fragments (direct global loads, rows past the chunk are zero)
    uint32_t qa[D / 16][4];
    const int r_lo = q0 + warp * 16 + g, r_hi = r_lo + 8;
    {
        const __nv_bfloat16 *qb = a.q + ((size_t)b * a.L) * a.ld_q + (size_t)h * D;
#pragma unroll
        for (int kk = 0; kk < D / 16; kk++) {
            const int c0 = kk * 16 + 2 * t4;
            qa[kk][0] = r_lo < a.L ? *reinterpret_cast<const uint32_t *>(qb + (size_t)r_lo * a.ld_q + c0) : 0u;
            qa[kk][1] = r_hi < a.L ? *reinterpret_cast<const uint32_t *>(qb + (size_t)r_hi * a.ld_q + c0) : 0u;
            qa[kk][2] = r_lo < a.L ? *reinterpret_cast<const uint32_t *>(qb + (size_t)r_lo * a.ld_q + c0 + 8) : 0u;
            qa[kk][3] = r_hi < a.L ? *reinterpret_cast<const uint32_t *>(qb + (size_t)r_hi * a.ld_q + c0 + 8) : 0u;
        }
    }
    const int pos_lo = a.p0 + r_lo, pos_hi = a.p0 + r_hi;
    const float sl2 = a.scale * 1.4426950408889634f;  // scores in log2 units

    float o[D / 8][4];
#pragma unroll
    for (int j = 0; j < D / 8; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;

    for (int kt = 0; kt < nkt; kt++) {
        const int buf = kt & 1;
        if (kt + 1 < nkt) {
            load_tile(kt + 1, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const uint32_t bk = smem_addr(sK + buf * kFaKeys * D * 2), bv = smem_addr(sV + buf * kFaKeys * D * 2);
        // ---- S = Q K^T (16 x 64 per warp) ----
        float s[kFaKeys / 8][4];
#pragma unroll
        for (int j = 0; j < kFaKeys / 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < D / 16; kk++) {
#pragma unroll
            for (int nj = 0; nj < kFaKeys / 16; nj++) {
                const int i = lane >> 3;
                const int key = nj * 16 + (i >> 1) * 8 + (lane & 7);
                const int ch = kk * 2 + (i & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(bk + fa_off<D>(key, ch), b0, b1, b2, b3);
                mma_bf16(s[2 * nj], qa[kk], b0, b1);
                mma_bf16(s[2 * nj + 1], qa[kk], b2, b3);
            }
        }
        // ---- causal mask + online softmax ----
        const int kbase = kt * kFaKeys;
        float mx_lo = m_lo, mx_hi = m_hi;
#pragma unroll
        for (int j = 0; j < kFaKeys / 8; j++) {
            const int k0 = kbase + j * 8 + 2 * t4;
            s[j][0] = k0 <= pos_lo ? s[j][0] * sl2 : -INFINITY;
            s[j][1] = k0 + 1 <= pos_lo ? s[j][1] * sl2 : -INFINITY;
            s[j][2] = k0 <= pos_hi ? s[j][2] * sl2 : -INFINITY;
            s[j][3] = k0 + 1 <= pos_hi ? s[j][3] * sl2 : -INFINITY;
            mx_lo = fmaxf(mx_lo, fmaxf(s[j][0], s[j][1]));
            mx_hi = fmaxf(mx_hi, fmaxf(s[j][2], s[j][3]));
        }
#pragma unroll
        for (int off = 1; off < 4; off <<= 1) {
            mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, off));
            mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, off));
        }
        const float base_lo = mx_lo == -INFINITY ? 0.f : mx_lo, base_hi = mx_hi == -INFINITY ? 0.f : mx_hi;
        const float al_lo = exp2f(m_lo - base_lo), al_hi = exp2f(m_hi - base_hi);
        m_lo = mx_lo; m_hi = mx_hi;
        float sum_lo = 0.f, sum_hi = 0.f;
#pragma unroll
        for (int j = 0; j < kFaKeys / 8; j++) {
            s[j][0] = exp2f(s[j][0] - base_lo); s[j][1] = exp2f(s[j][1] - base_lo);
            s[j][2] = exp2f(s[j][2] - base_hi); s[j][3] = exp2f(s[j][3] - base_hi);
            sum_lo += s[j][0] + s[j][1];
            sum_hi += s[j][2] + s[j][3];
        }
        l_lo = l_lo * al_lo + sum_lo;
        l_hi = l_hi * al_hi + sum_hi;
#pragma unroll
        for (int j = 0; j < D / 8; j++) {
            o[j][0] *= al_lo; o[j][1] *= al_lo; o[j][2] *= al_hi; o[j][3] *= al_hi;
        }
        // ---- O += P V ----
#pragma unroll
        for (int kk = 0; kk < kFaKeys / 16; kk++) {
            uint32_t pa[4];
            pa[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
            pa[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
            pa[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
            pa[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int nj = 0; nj < D / 16; nj++) {
                const int i = lane >> 3;
                const int key = kk * 16 + (i & 1) * 8 + (lane & 7);
                const int ch = nj * 2 + (i >> 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(bv + fa_off<D>(key, ch), b0, b1, b2, b3);
                mma_bf16(o[2 * nj], pa, b0, b1);
                mma_bf16(o[2 * nj + 1], pa, b2, b3);
            }
        }
        __syncthreads();  // this buffer is refilled by the next iteration's prefetch
    }
    // ---- normalise and store ----
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
        l_lo += __shfl_xor_sync(0xffffffffu, l_lo, off);
        l_hi += __shfl_xor_sync(0xffffffffu, l_hi, off);
    }
    const float inv_lo = l_lo > 0.f ? 1.0f / l_lo : 0.f, inv_hi = l_hi > 0.f ? 1.0f / l_hi : 0.f;
    __nv_bfloat16 *ob = a.out + ((size_t)b * a.L) * a.ld_out + (size_t)h * D;
#pragma unroll
    for (int j = 0; j < D / 8; j++) {
        const int c = j * 8 + 2 * t4;
        if (r_lo < a.L) *reinterpret_cast<uint32_t *>(ob + (size_t)r_lo * a.ld_out + c) = pack_bf16(o[j][0] * inv_lo, o[j][1] * inv_lo);
        if (r_hi < a.L) *reinterpret_cast<uint32_t *>(ob + (size_t)r_hi * a.ld_out + c) = pack_bf16(o[j][2] * inv_hi, o[j][3] * inv_hi);
    }
}

cudaError_t flash_prefill_launch(const FlashArgs &a, int nseq, cudaStream_t st) {
    dim3 grid((a.L + kFaRows - 1) / kFaRows, a.H, nseq);
    if (a.d == 128) {
        const size_t smem = 4 * kFaKeys * 128 * 2;
        return launch_pdl(qw_flash_prefill_kernel<128>, grid, dim3(kFaWarps * 32), smem, st, a);
    }
    if (a.d == 64) return launch_pdl(qw_flash_prefill_kernel<64>, grid, dim3(kFaWarps * 32), 4 * kFaKeys * 64 * 2, st, a);
    return cudaErrorInvalidValue;
}


// ------------------------------------------------------------------------------------------
// flash_decode: one query token per sequence, the G query heads of a KV head as the rows of
// one 16-row mma tile.  Grid (splits of the context, KV heads, sequences), 4 warps; every
// 64-key tile is staged by cp.async (3 stages) and each warp takes 16 of its keys with its own
// online-softmax state; warps, then splits (last CTA of each sequence / KV head), are merged.
// ------------------------------------------------------------------------------------------
constexpr int kFdStages = 3;

// byte offset of (row, 16-byte chunk) in a TMA-loaded [D / 64][64 rows][128 B] tile with the 128-byte swizzle
__device__ __forceinline__ uint32_t fd_off(int row, int chunk) {
    return (uint32_t)((chunk >> 3) * (kFaKeys * 128) + row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}

template <int D, int G>
__global__ void __launch_bounds__(kFaWarps * 32) qw_flash_decode_kernel(const __grid_constant__ CUtensorMap tmK,
                                                                         const __grid_constant__ CUtensorMap tmV,
                                                                         FlashDecodeArgs a) {
    griddep_launch_dependents();  // programmatic launch: the next kernel may start its prologue
    griddep_wait();               // the previous kernel's results
    constexpr int TILE_BYTES = kFaKeys * D * 2;
    extern __shared__ __align__(128) uint8_t fsm_raw[];
    // stages of [K tile | V tile], 1024-byte aligned for the swizzled TMA boxes
    uint8_t *fsm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(fsm_raw) + 1023) & ~(uintptr_t)1023);
    __shared__ __align__(8) uint64_t fd_full[kFdStages];
    __shared__ int fd_abort;
    __shared__ float wm[kFaWarps][16], wl[kFaWarps][16];
    __shared__ float sw[G][kFaMaxSplit];
    __shared__ int s_last;
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const int slot = a.slots ? a.slots[b] : b;
    const int pos = a.positions[b];
    const int n = pos + 1;
    const int ntile_all = (n + kFaKeys - 1) / kFaKeys;
    const int tiles_per = (ntile_all + a.nsplit - 1) / a.nsplit;
    const int kt0 = split * tiles_per, kt1 = min(ntile_all, kt0 + tiles_per);
    const int *ptab = a.page_table + (size_t)slot * a.max_pages;
    const __nv_bfloat16 *kc = reinterpret_cast<const __nv_bfloat16 *>(a.kcache);
    const __nv_bfloat16 *vc = reinterpret_cast<const __nv_bfloat16 *>(a.vcache);
    const int H = a.H, Hkv = a.Hkv;

    if (tid == 0) {
        for (int i = 0; i < kFdStages; i++) mbar_init(&fd_full[i], 1);
        fd_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmK) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmV) : "memory");
    }
    __syncthreads();
    volatile int *abort_flag = &fd_abort;
    // K and V rows [kt * 64, kt * 64 + 64) of this KV head: boxes of min(page, 64) rows x 64 columns from the
    // paged cache by TMA (one thread, no multicast); boxes past the last key read the zero fill
    const int br = a.page_size < kFaKeys ? a.page_size : kFaKeys;
    auto load_tile = [&](int kt, int st) {
        if (tid != 0) return;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // earlier reads of the stage are done
        uint8_t *bk = fsm + st * 2 * TILE_BYTES, *bv = bk + TILE_BYTES;
        mbar_arrive_expect_tx(&fd_full[st], 2 * TILE_BYTES);
        for (int r = 0; r < kFaKeys; r += br) {
            const int p = kt * kFaKeys + r;
            const int y = p < n ? (ptab[p >> a.log2_page] * Hkv + kvh) * a.page_size + (p & (a.page_size - 1)) : -br;
            for (int c = 0; c < D / 64; c++) {
                tma_load_2d(bk + c * kFaKeys * 128 + r * 128, &tmK, &fd_full[st], c * 64, y);
                tma_load_2d(bv + c * kFaKeys * 128 + r * 128, &tmV, &fd_full[st], c * 64, y);
            }
        }
    };

    float o[D / 8][4];
#pragma unroll
    for (int j = 0; j < D / 8; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;

    if (kt0 < kt1) {
        // prologue: the first stages (the KV rows written by earlier kernels)
        for (int i = 0; i < kFdStages - 1; i++)
            if (kt0 + i < kt1) load_tile(kt0 + i, i);
        // this warp's query rows: head kvh*G + row for row < G
        uint32_t qa[D / 16][4];
        {
            const __nv_bfloat16 *qb = a.q + (size_t)b * a.ld_q + (size_t)kvh * G * D;
#pragma unroll
            for (int kk = 0; kk < D / 16; kk++) {
                const int c0 = kk * 16 + 2 * t4;
                qa[kk][0] = g < G ? *reinterpret_cast<const uint32_t *>(qb + (size_t)g * D + c0) : 0u;
                qa[kk][2] = g < G ? *reinterpret_cast<const uint32_t *>(qb + (size_t)g * D + c0 + 8) : 0u;
                qa[kk][1] = 0u;  // rows 8..15 are padding (G <= 8)
                qa[kk][3] = 0u;
            }
        }
        const float sl2 = a.scale * 1.4426950408889634f;
        for (int kt = kt0; kt < kt1; kt++) {
            const int st = (kt - kt0) % kFdStages;
            if (kt + kFdStages - 1 < kt1) load_tile(kt + kFdStages - 1, (kt - kt0 + kFdStages - 1) % kFdStages);
            mbar_wait(&fd_full[st], (uint32_t)((kt - kt0) / kFdStages) & 1u, abort_flag, a.err);
            const uint32_t bk = smem_addr(fsm + st * 2 * TILE_BYTES), bv = bk + TILE_BYTES;
            float s[2][4];
            s[0][0] = s[0][1] = s[0][2] = s[0][3] = 0.f;
            s[1][0] = s[1][1] = s[1][2] = s[1][3] = 0.f;
#pragma unroll
            for (int kk = 0; kk < D / 16; kk++) {
                const int i = lane >> 3;
                const int key = warp * 16 + (i >> 1) * 8 + (lane & 7);
                const int ch = kk * 2 + (i & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(bk + fd_off(key, ch), b0, b1, b2, b3);
                mma_bf16(s[0], qa[kk], b0, b1);
                mma_bf16(s[1], qa[kk], b2, b3);
            }
            const int kbase = kt * kFaKeys + warp * 16;
            float mx_lo = m_lo, mx_hi = m_hi;
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const int k0 = kbase + j * 8 + 2 * t4;
                s[j][0] = k0 < n ? s[j][0] * sl2 : -INFINITY;
                s[j][1] = k0 + 1 < n ? s[j][1] * sl2 : -INFINITY;
                s[j][2] = k0 < n ? s[j][2] * sl2 : -INFINITY;
                s[j][3] = k0 + 1 < n ? s[j][3] * sl2 : -INFINITY;
                mx_lo = fmaxf(mx_lo, fmaxf(s[j][0], s[j][1]));
                mx_hi = fmaxf(mx_hi, fmaxf(s[j][2], s[j][3]));
            }
#pragma unroll
            for (int off = 1; off < 4; off <<= 1) {
                mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, off));
                mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, off));
            }
            const float base_lo = mx_lo == -INFINITY ? 0.f : mx_lo, base_hi = mx_hi == -INFINITY ? 0.f : mx_hi;
            const float al_lo = exp2f(m_lo - base_lo), al_hi = exp2f(m_hi - base_hi);
            m_lo = mx_lo; m_hi = mx_hi;
#pragma unroll
            for (int j = 0; j < 2; j++) {
                s[j][0] = exp2f(s[j][0] - base_lo); s[j][1] = exp2f(s[j][1] - base_lo);
                s[j][2] = exp2f(s[j][2] - base_hi); s[j][3] = exp2f(s[j][3] - base_hi);
            }
            l_lo = l_lo * al_lo + s[0][0] + s[0][1] + s[1][0] + s[1][1];
            l_hi = l_hi * al_hi + s[0][2] + s[0][3] + s[1][2] + s[1][3];
            uint32_t pa[4];
            pa[0] = pack_bf16(s[0][0], s[0][1]);
            pa[1] = pack_bf16(s[0][2], s[0][3]);
            pa[2] = pack_bf16(s[1][0], s[1][1]);
            pa[3] = pack_bf16(s[1][2], s[1][3]);
#pragma unroll
            for (int nj = 0; nj < D / 16; nj++) {
                const int i = lane >> 3;
                const int key = warp * 16 + (i & 1) * 8 + (lane & 7);
                const int ch = nj * 2 + (i >> 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(bv + fd_off(key, ch), b0, b1, b2, b3);
                o[2 * nj][0] *= al_lo; o[2 * nj][1] *= al_lo; o[2 * nj][2] *= al_hi; o[2 * nj][3] *= al_hi;
                o[2 * nj + 1][0] *= al_lo; o[2 * nj + 1][1] *= al_lo;
                o[2 * nj + 1][2] *= al_hi; o[2 * nj + 1][3] *= al_hi;
                mma_bf16(o[2 * nj], pa, b0, b1);
                mma_bf16(o[2 * nj + 1], pa, b2, b3);
            }
            __syncthreads();  // stage st is refilled by a later iteration
        }
        if (*abort_flag && tid == 0) {
            // a wait gave up: let the copies still in flight land before the shared memory is released
            const unsigned long long t0 = clock64();
            for (int st = 0; st < kFdStages; st++) {
                int last = -1;
                for (int kt = kt0; kt < kt1; kt++)
                    if ((kt - kt0) % kFdStages == st) last = kt;
                if (last < 0) continue;
                while (!mbar_try(smem_u32(&fd_full[st]), (uint32_t)((last - kt0) / kFdStages) & 1u) &&
                       (unsigned long long)clock64() - t0 < kTcuWaitCycles) {
                }
            }
        }
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) l_lo += __shfl_xor_sync(0xffffffffu, l_lo, off);
    (void)l_hi;
    (void)m_hi;

    // ---- merge the 4 warps (rows 0..G-1 only) through shared memory ----
    __syncthreads();
    float *so = reinterpret_cast<float *>(fsm);  // [warp][G][D]
    if (t4 == 0 && g < G) { wm[warp][g] = m_lo; wl[warp][g] = l_lo; }
    if (g < G) {
#pragma unroll
        for (int j = 0; j < D / 8; j++) {
            const int c = j * 8 + 2 * t4;
            so[((size_t)warp * G + g) * D + c] = o[j][0];
            so[((size_t)warp * G + g) * D + c + 1] = o[j][1];
        }
    }
    __syncthreads();
    for (int i = tid; i < G * D; i += kFaWarps * 32) {
        const int r = i / D, c = i % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kFaWarps; w++) M = fmaxf(M, wm[w][r]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kFaWarps; w++) {
                const float e = exp2f(wm[w][r] - M);
                L += wl[w][r] * e;
                O += so[((size_t)w * G + r) * D + c] * e;
            }
        }
        const int h = kvh * G + r;
        if (a.nsplit == 1) {
            a.out[(size_t)b * a.ld_out + (size_t)h * D + c] = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
        } else {
            const size_t pidx = ((size_t)b * H + h) * a.nsplit + split;
            a.part_o[pidx * D + c] = O;
            if (c == 0) { a.part_ml[pidx * 2] = M; a.part_ml[pidx * 2 + 1] = L; }
        }
    }
    if (a.nsplit == 1) return;

    // ---- split merge by the last CTA of this (sequence, KV head) ----
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(a.counters + (size_t)b * Hkv + kvh, 1u) == (unsigned)a.nsplit - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const size_t hb = (size_t)b * H + (size_t)kvh * G;
    if (tid < G) {
        float M = -INFINITY;
        for (int sp = 0; sp < a.nsplit; sp++) M = fmaxf(M, __ldcg(a.part_ml + ((hb + tid) * a.nsplit + sp) * 2));
        float L = 0.f;
        for (int sp = 0; sp < a.nsplit; sp++) {
            const float pm = __ldcg(a.part_ml + ((hb + tid) * a.nsplit + sp) * 2);
            const float e = (M == -INFINITY || pm == -INFINITY) ? 0.f : exp2f(pm - M);
            L += __ldcg(a.part_ml + ((hb + tid) * a.nsplit + sp) * 2 + 1) * e;
            sw[tid][sp] = e;
        }
        for (int sp = 0; sp < a.nsplit; sp++) sw[tid][sp] = L > 0.f ? sw[tid][sp] / L : 0.f;
    }
    __syncthreads();
    for (int i = tid; i < G * D; i += kFaWarps * 32) {
        const int r = i / D, c = i % D;
        const float *po = a.part_o + (hb + r) * a.nsplit * D + c;
        float O = 0.f;
        for (int sp = 0; sp < a.nsplit; sp++) O += sw[r][sp] * __ldcg(po + (size_t)sp * D);
        a.out[(size_t)b * a.ld_out + (size_t)(kvh * G + r) * D + c] = __float2bfloat16_rn(O);
    }
    if (tid == 0) a.counters[(size_t)b * Hkv + kvh] = 0u;
}

template <int D>
static cudaError_t flash_decode_g(const FlashDecodeArgs &a, dim3 grid, cudaStream_t st) {
    const size_t smem = (size_t)kFdStages * 2 * kFaKeys * D * 2 + 1024;
    const dim3 block(kFaWarps * 32);
    CUtensorMap mk, mv;
    const long long rows = (long long)a.num_pages * a.Hkv * a.page_size;
    const int br = a.page_size < kFaKeys ? a.page_size : kFaKeys;
    cudaError_t e = tma_map_bf16_sw128(&mk, a.kcache, rows, D, D, br);
    if (e != cudaSuccess) return e;
    e = tma_map_bf16_sw128(&mv, a.vcache, rows, D, D, br);
    if (e != cudaSuccess) return e;
    switch (a.H / a.Hkv) {
        case 1: return launch_pdl(qw_flash_decode_kernel<D, 1>, grid, block, smem, st, mk, mv, a);
        case 2: return launch_pdl(qw_flash_decode_kernel<D, 2>, grid, block, smem, st, mk, mv, a);
        case 4: return launch_pdl(qw_flash_decode_kernel<D, 4>, grid, block, smem, st, mk, mv, a);
        case 6: return launch_pdl(qw_flash_decode_kernel<D, 6>, grid, block, smem, st, mk, mv, a);
        case 7: return launch_pdl(qw_flash_decode_kernel<D, 7>, grid, block, smem, st, mk, mv, a);
        case 8: return launch_pdl(qw_flash_decode_kernel<D, 8>, grid, block, smem, st, mk, mv, a);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t flash_decode_launch(const FlashDecodeArgs &a, int B, cudaStream_t st) {
    if (a.nsplit < 1 || a.nsplit > kFaMaxSplit) return cudaErrorInvalidValue;
    dim3 grid(a.nsplit, a.Hkv, B);
    if (a.d == 128) return flash_decode_g<128>(a, grid, st);
    if (a.d == 64) return flash_decode_g<64>(a, grid, st);
    return cudaErrorInvalidValue;
}

// ------------------------------------------------------------------------------------------
// rows_argmax: one CTA per logits row; first index of the maximum
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(512) qw_rows_argmax_kernel(RowsArgmaxArgs a) {
    griddep_launch_dependents();  // programmatic launch: the next kernel may start its prologue
    griddep_wait();               // the previous kernel's results
    __shared__ float sv[16];
    __shared__ int si[16];
    const int b = blockIdx.x, tid = threadIdx.x;
    const float *row = a.logits + (size_t)b * a.ld;
    float bv = -FLT_MAX;
    int bi = INT_MAX;
    if (a.cand_val) {
        const float *cv = a.cand_val + (size_t)b * a.ld;
        const int *ci = a.cand_idx + (size_t)b * a.ld;
        for (int i = tid; i < a.n; i += blockDim.x) {
            const float v = cv[i];
            const int ix = ci[i];
            if (v > bv || (v == bv && ix < bi)) { bv = v; bi = ix; }
        }
    } else {
        for (int i = tid; i < a.n; i += blockDim.x) {
            const float v = row[i];
            if (v > bv) { bv = v; bi = i; }  // increasing i per thread: strict > keeps the first
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if ((tid & 31) == 0) { sv[tid >> 5] = bv; si[tid >> 5] = bi; }
    __syncthreads();
    if (tid == 0) {
        bv = sv[0]; bi = si[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); w++)
            if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
        const int gidx = bi + a.idx_offset;
        if (a.argmax_val) a.argmax_val[b] = bv;
        if (a.argmax_out) a.argmax_out[b] = gidx;
        if (a.hist) a.hist[(size_t)b * a.hist_ld + a.positions[b] + 1] = gidx;
        if (a.advance) {
            a.next_tokens[b] = gidx;
            a.positions[b] += 1;
        }
    }
}

cudaError_t prefill_kernels_prepare() {
    const void *fns[] = {(const void *)qw_norm_rows_kernel, (const void *)qw_qkv_post_kernel<__nv_bfloat16>,
                         (const void *)qw_qkv_post_kernel<float>, (const void *)qw_flash_prefill_kernel<128>,
                         (const void *)qw_flash_prefill_kernel<64>,
                         (const void *)qw_flash_decode_kernel<128, 1>, (const void *)qw_flash_decode_kernel<128, 2>,
                         (const void *)qw_flash_decode_kernel<128, 4>, (const void *)qw_flash_decode_kernel<128, 8>,
                         (const void *)qw_flash_decode_kernel<128, 6>, (const void *)qw_flash_decode_kernel<128, 7>,
                         (const void *)qw_flash_decode_kernel<64, 6>, (const void *)qw_flash_decode_kernel<64, 7>,
                         (const void *)qw_flash_decode_kernel<64, 1>, (const void *)qw_flash_decode_kernel<64, 2>,
                         (const void *)qw_flash_decode_kernel<64, 4>, (const void *)qw_flash_decode_kernel<64, 8>};
    for (const void *f : fns) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPrepSmem);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t rows_argmax_launch(const RowsArgmaxArgs &a, int rows, cudaStream_t st) {
    return launch_pdl(qw_rows_argmax_kernel, dim3(rows), dim3(512), 0, st, a);
}

}  // namespace qw

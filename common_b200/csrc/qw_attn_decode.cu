// qw_attn_decode.cu -- decode-time GQA attention over the paged KV cache.
//
// One CTA per (split of the context, KV head, sequence).  The prologue does, for the
// query heads of its KV group and for that KV head:
//   QK-norm   whole-vector rmsnorm (the reference: AttentionFeatures.java:840-845, 886-891)
//             or per-head rmsnorm (HF Qwen3), eps 1e-6;
//   RoPE      split-half rotation with the (position, f) cos/sin table
//             (AttentionFeatures.java:195-237, RotationFeatures.java:124-170, 189-208);
//   KV write  split 0 stores this position's k and v into the paged cache.  The reference
//             stores GQA-expanded rows (seqLen, heads, headSize) (AttentionFeatures.java:823-826,
//             372-391); here each KV head is stored once and shared by its query heads, which
//             reads the same values.
// The main loop streams K and V rows of the CTA's token range with the online
// (running max / running sum) form of the log-stable softmax of ActivationFeatures.java:136-142
// over scores q.k/sqrt(d) (AttentionFeatures.java:531-559) and accumulates p.V
// (AttentionFeatures.java:572-616).  Positions after the current one carry the reference's
// -10000 mask (AttentionFeatures.java:906-917), whose softmax weight is exactly 0 in fp32/fp64,
// so they are skipped.  Splits are merged by the last CTA of each (sequence, KV head).
#include "qw_internal.cuh"
#include <math.h>

namespace qw {

constexpr int kAttnWarps = 8;
constexpr int kAttnTPW = 8;  // tokens per warp per tile: a tile is 64 tokens
constexpr int kAttnMaxSplit = 64;

// per-lane slice (DPL elements) of one K or V row, kept packed in registers until used
template <typename KT, int DPL> struct KVec;
template <> struct KVec<__nv_bfloat16, 4> {
    using T = uint2;
    static __device__ __forceinline__ T load(const __nv_bfloat16 *p) { return *reinterpret_cast<const uint2 *>(p); }
    static __device__ __forceinline__ void unpack(const T &u, float *f) {
        f[0] = bf16lo(u.x); f[1] = bf16hi(u.x); f[2] = bf16lo(u.y); f[3] = bf16hi(u.y);
    }
};
template <> struct KVec<__nv_bfloat16, 2> {
    using T = uint32_t;
    static __device__ __forceinline__ T load(const __nv_bfloat16 *p) { return *reinterpret_cast<const uint32_t *>(p); }
    static __device__ __forceinline__ void unpack(const T &u, float *f) { f[0] = bf16lo(u); f[1] = bf16hi(u); }
};
template <> struct KVec<float, 4> {
    using T = float4;
    static __device__ __forceinline__ T load(const float *p) { return *reinterpret_cast<const float4 *>(p); }
    static __device__ __forceinline__ void unpack(const T &u, float *f) { f[0] = u.x; f[1] = u.y; f[2] = u.z; f[3] = u.w; }
};
template <> struct KVec<float, 2> {
    using T = float2;
    static __device__ __forceinline__ T load(const float *p) { return *reinterpret_cast<const float2 *>(p); }
    static __device__ __forceinline__ void unpack(const T &u, float *f) { f[0] = u.x; f[1] = u.y; }
};

__device__ __forceinline__ float block_sum(float v, float *scratch) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; w++) s += scratch[w];
    return s;
}

template <typename KT, int D, int G, int DPL>
__device__ __forceinline__ void attn_issue(typename KVec<KT, DPL>::T (&kr)[kAttnTPW], typename KVec<KT, DPL>::T (&vr)[kAttnTPW],
                                           const KT *kc, const KT *vc, const int *ptab, int tbase, int t1, int pos,
                                           int Hkv, int kvh, int ps, int lg, int warp, int lane) {
#pragma unroll
    for (int j = 0; j < kAttnTPW; j++) {
        const int tt = tbase + warp * kAttnTPW + j;
        if (tt < t1 && tt != pos) {
            size_t base = (((size_t)ptab[tt >> lg] * Hkv + kvh) * ps + (tt & (ps - 1))) * D + lane * DPL;
            kr[j] = KVec<KT, DPL>::load(kc + base);
            vr[j] = KVec<KT, DPL>::load(vc + base);
        }
    }
}

template <typename KT, int D, int G>
__global__ void __launch_bounds__(kAttnWarps * 32) qw_attn_decode_kernel(const AttnArgs a) {
    constexpr int DPL = D / 32;
    constexpr int HALF = D / 2;
    constexpr int TILE = kAttnWarps * kAttnTPW;
    using KV = KVec<KT, DPL>;
    __shared__ __align__(16) float qs[G][D];
    __shared__ __align__(16) float ks[D];
    __shared__ __align__(16) float vs[D];
    __shared__ float wm[kAttnWarps][G], wl[kAttnWarps][G];
    __shared__ __align__(16) float wo[kAttnWarps][G][D];
    __shared__ float scratch[kAttnWarps];
    __shared__ float s_scale[2];
    __shared__ int s_last;

    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int H = a.H, Hkv = a.Hkv;
    // positions / slots / page table were written at least two kernels earlier, which have
    // completed before this grid can start (every kernel triggers its dependents only after its
    // own wait), so they may be read before the wait below.
    const int slot = a.slots ? a.slots[b] : b;
    const int pos = a.positions[b];
    // token range of this split: at least 64 tokens per split, so short contexts use few splits
    const int n = pos + 1;
    int chunk = (n + a.nsplit - 1) / a.nsplit;
    chunk = chunk < TILE ? TILE : chunk;
    const int ns_eff = (n + chunk - 1) / chunk;
    const int t0 = split * chunk;
    const int t1 = min(n, t0 + chunk);
    const int *ptab = a.page_table + (size_t)slot * a.max_pages;
    const int ps = a.page_size, lg = a.log2_page;
    KT *kc = reinterpret_cast<KT *>(a.kcache);
    KT *vc = reinterpret_cast<KT *>(a.vcache);

    typename KV::T kr[kAttnTPW], vr[kAttnTPW], kn[kAttnTPW], vn[kAttnTPW];
    // the cached K/V rows do not depend on the previous kernel: start loading them now
    if (t0 < n) attn_issue<KT, D, G, DPL>(kr, vr, kc, vc, ptab, t0, t1, pos, Hkv, kvh, ps, lg, warp, lane);
    griddep_wait();
    griddep_launch_dependents();

    if (t0 < n) {
    const float *row = a.qkv + (size_t)b * a.ld_qkv;
    const float *qrow = row + (size_t)kvh * G * D;
    const float *krow = row + (size_t)H * D + (size_t)kvh * D;
    const float *vrow = row + (size_t)(H + Hkv) * D + (size_t)kvh * D;

    for (int i = tid; i < G * D; i += blockDim.x) qs[i / D][i % D] = qrow[i];
    for (int i = tid; i < D; i += blockDim.x) { ks[i] = krow[i]; vs[i] = vrow[i]; }

    // ---------------- QK-norm ----------------
    if (a.qk_mode == 1) {
        if (a.qk_ss) {
            if (tid == 0) {
                s_scale[0] = 1.0f / sqrtf(a.qk_ss[b * 2 + 0] / (float)a.q_total + 1e-6f);
                s_scale[1] = 1.0f / sqrtf(a.qk_ss[b * 2 + 1] / (float)a.kv_total + 1e-6f);
            }
        } else {
            float sq = 0.f, sk = 0.f;
#pragma unroll 8
            for (int i = tid; i < H * D; i += blockDim.x) sq += row[i] * row[i];
#pragma unroll 4
            for (int i = tid; i < Hkv * D; i += blockDim.x) sk += row[H * D + i] * row[H * D + i];
            sq = block_sum(sq, scratch);
            sk = block_sum(sk, scratch);
            if (tid == 0) {
                s_scale[0] = 1.0f / sqrtf(sq / (float)a.q_total + 1e-6f);
                s_scale[1] = 1.0f / sqrtf(sk / (float)a.kv_total + 1e-6f);
            }
        }
        __syncthreads();
        const float sq = s_scale[0], sk = s_scale[1];
        for (int i = tid; i < G * D; i += blockDim.x) {
            int g = i / D, j = i % D;
            qs[g][j] = a.qn[(size_t)(kvh * G + g) * D + j] * qs[g][j] * sq;
        }
        for (int i = tid; i < D; i += blockDim.x) ks[i] = a.kn[(size_t)kvh * D + i] * ks[i] * sk;
    } else if (a.qk_mode == 2) {
        __syncthreads();
        // one warp per head (G query heads + 1 key head)
        for (int hh = warp; hh <= G; hh += kAttnWarps) {
            float *v = hh < G ? qs[hh] : ks;
            const float *w = hh < G ? a.qn + (size_t)(kvh * G + hh) * D : a.kn + (size_t)kvh * D;
            float s = 0.f;
            for (int i = lane; i < D; i += 32) s += v[i] * v[i];
            s = warp_sum(s);
            float sc = 1.0f / sqrtf(s / (float)D + 1e-6f);
            for (int i = lane; i < D; i += 32) v[i] = w[i] * v[i] * sc;
        }
    }
    __syncthreads();

    // ---------------- RoPE (split-half) ----------------
    const float2 *fr = a.freq + (size_t)pos * HALF;
    for (int i = tid; i < (G + 1) * HALF; i += blockDim.x) {
        int hh = i / HALF, f = i % HALF;
        float *v = hh < G ? qs[hh] : ks;
        float2 cs = fr[f];
        float x1 = v[f], x2 = v[f + HALF];
        v[f] = x1 * cs.x - x2 * cs.y;
        v[f + HALF] = x2 * cs.x + x1 * cs.y;
    }
    __syncthreads();
    // the cached row is stored in KT; use the rounded values for this position too
    for (int i = tid; i < D; i += blockDim.x) { ks[i] = Elt<KT>::round(ks[i]); vs[i] = Elt<KT>::round(vs[i]); }
    __syncthreads();

    if (split == 0) {
        size_t base = (((size_t)ptab[pos >> lg] * Hkv + kvh) * ps + (pos & (ps - 1))) * D;
        for (int i = tid; i < D; i += blockDim.x) {
            Elt<KT>::store(kc + base + i, ks[i]);
            Elt<KT>::store(vc + base + i, vs[i]);
        }
    }

    // ---------------- main loop: 64-token tiles, next tile's loads in flight ----------------
    float qreg[G][DPL];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int j = 0; j < DPL; j++) qreg[g][j] = qs[g][lane * DPL + j] * a.scale;
    float m[G], l[G], o[G][DPL];
#pragma unroll
    for (int g = 0; g < G; g++) {
        m[g] = -INFINITY; l[g] = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; j++) o[g][j] = 0.f;
    }
    float kcur[DPL], vcur[DPL];
#pragma unroll
    for (int j = 0; j < DPL; j++) { kcur[j] = ks[lane * DPL + j]; vcur[j] = vs[lane * DPL + j]; }

    for (int tb = t0; tb < t1; tb += TILE) {
        if (tb + TILE < t1) attn_issue<KT, D, G, DPL>(kn, vn, kc, vc, ptab, tb + TILE, t1, pos, Hkv, kvh, ps, lg, warp, lane);
        float sc[kAttnTPW][G];
#pragma unroll
        for (int j = 0; j < kAttnTPW; j++) {
            const int tt = tb + warp * kAttnTPW + j;
            float kf[DPL];
            if (tt == pos) {
#pragma unroll
                for (int e = 0; e < DPL; e++) kf[e] = kcur[e];
            } else {
                KV::unpack(kr[j], kf);
            }
#pragma unroll
            for (int g = 0; g < G; g++) {
                float sacc = 0.f;
#pragma unroll
                for (int e = 0; e < DPL; e++) sacc = fmaf(qreg[g][e], kf[e], sacc);
                sc[j][g] = tt < t1 ? warp_sum(sacc) : -INFINITY;
            }
        }
#pragma unroll
        for (int g = 0; g < G; g++) {
            float mx = m[g];
#pragma unroll
            for (int j = 0; j < kAttnTPW; j++) mx = fmaxf(mx, sc[j][g]);
            if (mx == -INFINITY) continue;  // this warp has no tokens in the tile
            const float alpha = expf(m[g] - mx);
            l[g] *= alpha;
#pragma unroll
            for (int e = 0; e < DPL; e++) o[g][e] *= alpha;
            m[g] = mx;
#pragma unroll
            for (int j = 0; j < kAttnTPW; j++) sc[j][g] = expf(sc[j][g] - mx);
        }
#pragma unroll
        for (int j = 0; j < kAttnTPW; j++) {
            const int tt = tb + warp * kAttnTPW + j;
            if (tt >= t1) continue;
            float vf[DPL];
            if (tt == pos) {
#pragma unroll
                for (int e = 0; e < DPL; e++) vf[e] = vcur[e];
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
#pragma unroll
        for (int j = 0; j < kAttnTPW; j++) { kr[j] = kn[j]; vr[j] = vn[j]; }
    }

    // ---------------- merge warps ----------------
#pragma unroll
    for (int g = 0; g < G; g++) {
        if (lane == 0) { wm[warp][g] = m[g]; wl[warp][g] = l[g]; }
#pragma unroll
        for (int j = 0; j < DPL; j++) wo[warp][g][lane * DPL + j] = o[g][j];
    }
    __syncthreads();
    for (int i = tid; i < G * D; i += blockDim.x) {
        int g = i / D, j = i % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttnWarps; w++) M = fmaxf(M, wm[w][g]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kAttnWarps; w++) {
                float e = expf(wm[w][g] - M);
                L += wl[w][g] * e;
                O += wo[w][g][j] * e;
            }
        }
        int h = kvh * G + g;
        if (a.nsplit == 1) {
            const size_t oi = (size_t)b * a.ld_out + (size_t)h * D + j;
            if (a.out_bf16) a.out_bf16[oi] = __float2bfloat16_rn(O / L);
            else a.out[oi] = O / L;
        } else {
            size_t pidx = ((size_t)b * H + h) * a.nsplit + split;
            a.part_o[pidx * D + j] = O;
            if (j == 0) { a.part_ml[pidx * 2 + 0] = M; a.part_ml[pidx * 2 + 1] = L; }
        }
    }
    }  // t0 < n
    if (a.nsplit == 1) return;

    // ---------------- split merge: the last CTA of this (sequence, KV head) ----------------
    __shared__ float sw[G][kAttnMaxSplit];
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        unsigned t = atomicAdd(a.counters + (size_t)b * Hkv + kvh, 1u);
        s_last = (t == (unsigned)a.nsplit - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const size_t hb = (size_t)b * H + (size_t)kvh * G;  // first head of this group
    for (int i = tid; i < G * ns_eff; i += blockDim.x) {
        int g = i / ns_eff, s = i % ns_eff;
        sw[g][s] = __ldcg(a.part_ml + ((hb + g) * a.nsplit + s) * 2);
    }
    __syncthreads();
    if (tid < G) {
        float M = -INFINITY;
        for (int s = 0; s < ns_eff; s++) M = fmaxf(M, sw[tid][s]);
        float L = 0.f;
        for (int s = 0; s < ns_eff; s++) {
            float e = expf(sw[tid][s] - M);
            L += __ldcg(a.part_ml + ((hb + tid) * a.nsplit + s) * 2 + 1) * e;
            sw[tid][s] = e;
        }
        for (int s = 0; s < ns_eff; s++) sw[tid][s] /= L;
    }
    __syncthreads();
    for (int i = tid; i < G * D; i += blockDim.x) {
        int g = i / D, j = i % D;
        const float *po = a.part_o + (hb + g) * a.nsplit * D + j;
        float O = 0.f;
#pragma unroll 4
        for (int s = 0; s < ns_eff; s++) O += sw[g][s] * __ldcg(po + (size_t)s * D);
        const size_t oi = (size_t)b * a.ld_out + (size_t)(kvh * G + g) * D + j;
        if (a.out_bf16) a.out_bf16[oi] = __float2bfloat16_rn(O);
        else a.out[oi] = O;
    }
    if (tid == 0) a.counters[(size_t)b * Hkv + kvh] = 0u;
}

template <typename KT, int D>
static cudaError_t attn_launch_g(const AttnArgs &a, int G, dim3 grid, cudaStream_t st) {
    switch (G) {
        case 1: qw_attn_decode_kernel<KT, D, 1><<<grid, kAttnWarps * 32, 0, st>>>(a); break;
        case 2: qw_attn_decode_kernel<KT, D, 2><<<grid, kAttnWarps * 32, 0, st>>>(a); break;
        case 4: qw_attn_decode_kernel<KT, D, 4><<<grid, kAttnWarps * 32, 0, st>>>(a); break;
        case 6: qw_attn_decode_kernel<KT, D, 6><<<grid, kAttnWarps * 32, 0, st>>>(a); break;
        case 7: qw_attn_decode_kernel<KT, D, 7><<<grid, kAttnWarps * 32, 0, st>>>(a); break;
        case 8: qw_attn_decode_kernel<KT, D, 8><<<grid, kAttnWarps * 32, 0, st>>>(a); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t attn_decode_launch(const AttnArgs &a, int B, bool kv_bf16, cudaStream_t st) {
    if (a.Hkv <= 0 || a.H % a.Hkv) return cudaErrorInvalidValue;
    int G = a.H / a.Hkv;
    dim3 grid(a.nsplit, a.Hkv, B);
    if (a.d == 128) return kv_bf16 ? attn_launch_g<__nv_bfloat16, 128>(a, G, grid, st) : attn_launch_g<float, 128>(a, G, grid, st);
    if (a.d == 64) return kv_bf16 ? attn_launch_g<__nv_bfloat16, 64>(a, G, grid, st) : attn_launch_g<float, 64>(a, G, grid, st);
    return cudaErrorInvalidValue;
}

}  // namespace qw

// qw_tc.h -- host interface of the tcgen05 / TMEM / TMA GEMM (qw_gemm.cu).
//
// out(t, f) = sum_k W(f, k) * X(t, k) for bf16 W (M, K) and X (T, K), both row-major (K
// contiguous), fp32 accumulation in tensor memory.  W is the MMA's M side (128 output
// features per tile) and the tokens are its N side (64, 128 or 256 per tile), so the same
// kernel serves prefill (T in the thousands) and batched decode (T = batch).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace qw {

enum TcEpi {
    TC_STORE = 0,   // out_f32[t * ld_out + f] = acc (+ bias[f])
    TC_RESID = 1,   // out_f32[t * ld_out + f] = resid[t * ld_resid + f] + acc
    TC_SWIGLU = 2,  // W rows interleaved 16 gate / 16 up: out_bf16[t * ld_out + pair] = up * silu(gate)
    TC_ARGMAX = 3,  // optional STORE (out may be null) and, per token and 32 features, the first maximum:
                    // cand_val / cand_idx[t * ncand + f / 32] (ncand >= 4 x 128-row tiles of M)
};

// device-side error codes written to TcArgs::err
enum { TC_DEVERR_TIMEOUT = 1 };

struct TcArgs {
    int M;       // output features (rows of W)
    int T;       // tokens (rows of X)
    int K;       // reduction length (multiple of 8)
    int ksplit;  // K ranges per output tile; > 1 accumulates with atomics (caller zeroes out, or out == resid)
    void *out;   // fp32 (STORE / RESID) or bf16 (SWIGLU)
    int ld_out;
    const float *resid;
    int ld_resid;
    const float *bias;  // STORE: optional (M)
    int *err;           // optional: set to TC_DEVERR_* when a bounded wait gives up
    float *cand_val;    // ARGMAX: (T, ncand) per-group maxima and their feature indices
    int *cand_idx;
    int ncand;
    int group_t;        // CTA-pair kernel: token tiles per group of its tile order (set by the launcher)
};

// Build the TMA descriptors and launch.  bn = 0 picks the token tile from T.
cudaError_t tc_gemm_launch(const void *W, const void *X, const TcArgs &a, int epi, int bn, int num_sms,
                           cudaStream_t st);

// TMA descriptor of a bf16 (rows, cols) row-major matrix with row stride ld elements: boxes of box_rows x 64
// columns (128 bytes), 128-byte swizzle, zero fill out of bounds.  base 16-byte aligned, ld a multiple of 8.
cudaError_t tma_map_bf16_sw128(CUtensorMap *m, const void *base, long long rows, int cols, int ld, int box_rows);

// Opt every GEMM variant in to its shared memory (once per device, outside of stream capture).
cudaError_t tc_prepare();

// K ranges per tile that fill the GPU for a skinny (decode) problem; 1 for large T.
int tc_pick_ksplit(int M, int T, int K, int bn, int num_sms);
int tc_pick_bn(int T);

}  // namespace qw

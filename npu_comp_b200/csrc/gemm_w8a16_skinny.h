// Internal interface of the stream-K W8A16 GEMM for few tokens
// (gemm_w8a16_skinny.cu).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace npub {

// Token counts up to this use the stream-K kernel (one token tile, BT = 32 or 64).
constexpr int kSkinnyMaxM = 64;

// An RMSNorm folded into the decode GEMMs (all fields null / zero: none).
//  * rs_part (consumer): the tokens A are fp16(h * gamma) of a residual stream
//    h; token t's result is multiplied by
//      1 / sqrt(sum_{i < rs_n} rs_part[i * rs_ld + t] / rs_d + rs_eps),
//    the partial sums of h^2 the producer wrote.
//  * gamma / G / ss (producer): besides C = fp16(acc * scale + R), store
//    G[t, n] = fp16(C[t, n] * gamma[n]) and, for every 32 consecutive output
//    columns n (chunk i = n / 32), ss[i * ss_ld + t] = sum of C[t, n]^2.
struct SkinnyNorm {
    const float* rs_part;
    int rs_n;
    int64_t rs_ld;
    float rs_d, rs_eps;
    const __half* gamma;
    __half* G;
    int64_t ldg;
    float* ss;
    int64_t ss_ld;
};

// The next stream-K GEMM of a chain (all null: none): its first weight tiles
// are prefetched to L2 once this kernel's own weights are requested.
struct SkinnyNext {
    const void* W;
    int64_t ldw;
    int M, N, K;
};

struct SkinnyParams {
    CUtensorMap tmW;  // int8 weights [N, K]: box {128, 128, 1}, 128-byte swizzle
    CUtensorMap tmX;  // fp16 activations [M, K]: box {64, BT, 1}, 128-byte swizzle
    int M, N, k_steps, n_tiles;
    __half* C;
    int64_t ldc;
    const __half* R;
    int64_t ldr;
    const __half* scale;
    float alpha;
    float* part;    // [grid][128][BT] fp32 partial tiles
    unsigned* cnt;  // [n_tiles][4] pieces arrived per tile and 32-row quarter (zero between calls)
    int* err;
    uint64_t wait_ns;  // limit of the waits on other CTAs' pieces
    int swiglu;     // 1: rows 2c / 2c+1 are gate / up; C [M, N/2] = fp16(silu(g) * u)
    SkinnyNorm nrm;
    int csplit;     // > 1: cluster split, grid = n_tiles * csplit (cluster t = tile t)
    CUtensorMap tmWn;  // the next GEMM's weights (pf_grid > 0)
    int pf_grid, pf_csplit, pf_tiles, pf_ksteps;
    int w_evict_first;  // weight loads marked evict-first in L2
    int r_stage;        // R staged in shared memory by 16-byte copies (R, ldr and N multiples of 8 halves)
};

// Tile counters at the start of every workspace of this kernel: a fixed
// region (never partial sums), 4 per 128-row tile, so N <= 524288.
constexpr size_t kSkinnyCounterBytes = 64 << 10;

// Whether (M, N) can run on the stream-K kernel, and whether it should.
bool w8a16_skinny_fits(int M, int N);
bool w8a16_use_skinny(int M, int N, int K);
size_t w8a16_skinny_workspace(int M, int N, int K);
int w8a16_skinny_run(const void* A, int64_t lda, const void* W, int64_t ldw, const void* scale, void* C, int64_t ldc,
                     const void* R, int64_t ldr, int M, int N, int K, float alpha, void* ws, size_t ws_bytes,
                     cudaStream_t st, int swiglu = 0, const SkinnyNorm* nrm = nullptr,
                     const SkinnyNext* next = nullptr);

}  // namespace npub

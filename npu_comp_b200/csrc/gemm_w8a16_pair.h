// Internal interface of the 2-CTA-pair W8A16 GEMM (gemm_w8a16_pair.cu).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace npub {

// TMA ring depths per token-tile width and the depth of the converted fp16
// weight ring; one stage carries kPairBK = 128 of K (48/32/24 KB of TMA data
// at BT = 256/128/64, 32 KB of converted weights).  Measured on B200: the
// per-stage synchronisation cost is fixed, so two 64-wide K chunks per stage
// beat deeper rings of single chunks (1113 vs 915 TFLOP/s at 2048x22016x4096).  The TMA
// depth must be even: the two converter groups take alternate K steps, and a
// group waiting for step g relies on having itself consumed step g - STAGES
// (so the barrier phase it waits on cannot alias an older one).
#ifndef NPUB_PAIR_STAGES256
#define NPUB_PAIR_STAGES256 3
#endif
#ifndef NPUB_PAIR_STAGES128
#define NPUB_PAIR_STAGES128 5
#endif
#ifndef NPUB_PAIR_STAGES64
#define NPUB_PAIR_STAGES64 4
#endif
#ifndef NPUB_PAIR_CSTAGES64
#define NPUB_PAIR_CSTAGES64 4
#endif
#ifndef NPUB_PAIR_GROUPS64
#define NPUB_PAIR_GROUPS64 2
#endif
#ifndef NPUB_PAIR_CSTAGES
#define NPUB_PAIR_CSTAGES 2
#endif
#ifndef NPUB_PAIR_CONV_GROUPS
#define NPUB_PAIR_CONV_GROUPS 1
#endif
constexpr int kPairStages256 = NPUB_PAIR_STAGES256;
constexpr int kPairStages128 = NPUB_PAIR_STAGES128;
constexpr int kPairStages64 = NPUB_PAIR_STAGES64;
constexpr int kPairCStages = NPUB_PAIR_CSTAGES;
constexpr int kPairConvGroups = NPUB_PAIR_CONV_GROUPS;  // converter groups of 4 warps (alternate K steps)
// Skinny (decode) tiles: the tensor core finishes a stage quickly, so the
// int8 -> fp16 conversion hand-off is the critical path; more converted stages
// and two converter groups keep it off.
constexpr int kPairCStages64 = NPUB_PAIR_CSTAGES64;
constexpr int kPairGroups64 = NPUB_PAIR_GROUPS64;
#ifndef NPUB_PAIR_KCH
#define NPUB_PAIR_KCH 2
#endif
// 64-wide K chunks per pipeline stage (one 128-byte swizzled row of fp16 each).
constexpr int kPairKch = NPUB_PAIR_KCH;
constexpr int kPairBK = 64 * kPairKch;

struct PairParams {
    CUtensorMap tmW;  // int8 weights [N, K]: box {64, 128, 1}, no swizzle
    CUtensorMap tmX;  // fp16 activations [M, K]: box {64, BT/2, 1}, 128-byte swizzle
    int M, N, k_tiles;
    int n_apairs, n_btiles, splits, k_tiles_per_split, n_tiles;
    int out_f32;            // 1: fp32 partials [splits, M, N] to `part` (no scale / residual)
    __half* C;
    int64_t ldc;
    const __half* R;
    int64_t ldr;
    const __half* scale;
    float alpha;
    float* part;
    int* err;
    int swiglu;             // 1: rows 2c / 2c+1 are gate / up; C [M, N/2] = fp16(silu(g) * u)
    int band;               // token tiles per band of the tile order (set by w8a16_pair_run)
};

int pair_bt(int M);
size_t w8a16_pair_workspace(int M, int N, int K);
int w8a16_pair_splits(int M, int N, int K);
int w8a16_pair_run(PairParams& p, int M, int N, int K, cudaStream_t st);

}  // namespace npub

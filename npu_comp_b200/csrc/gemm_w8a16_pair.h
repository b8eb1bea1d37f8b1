// Internal interface of the 2-CTA-pair W8A16 GEMM (gemm_w8a16_pair.cu).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace npub {

// TMA ring depths per token-tile width (shared memory: 24/16/12 KB per stage)
// and the depth of the converted fp16 weight ring (16 KB per stage).  The TMA
// depth must be even: the two converter groups take alternate K steps, and a
// group waiting for step g relies on having itself consumed step g - STAGES
// (so the barrier phase it waits on cannot alias an older one).
constexpr int kPairStages256 = 6;
constexpr int kPairStages128 = 10;
constexpr int kPairStages64 = 12;
constexpr int kPairCStages = 4;

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
};

int pair_bt(int M);
size_t w8a16_pair_workspace(int M, int N, int K);
int w8a16_pair_splits(int M, int N, int K);
int w8a16_pair_run(PairParams& p, int M, int N, int K, cudaStream_t st);

}  // namespace npub

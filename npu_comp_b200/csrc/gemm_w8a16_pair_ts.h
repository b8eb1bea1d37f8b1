// Internal interface of the prefill W8A16 GEMM with converted weights in
// tensor memory (gemm_w8a16_pair_ts.cu).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace npub {

struct PairTsParams {
    CUtensorMap tmW;  // int8 weights [N, K]: box {128, 128, 1}, 128-byte swizzle
    CUtensorMap tmX;  // fp16 activations [M, K]: box {64, 96, 1}, 128-byte swizzle
    int M, N, k_steps;
    int n_apairs, n_btiles, n_tiles;
    __half* C;
    int64_t ldc;
    const __half* R;
    int64_t ldr;
    const __half* scale;
    float alpha;
    int* err;
};

// True where the tensor-memory pair kernel is the W8A16 kernel of choice.
bool w8a16_use_pair_ts(int M, int N, int K);
int w8a16_pair_ts_run(const void* A, int64_t lda, const void* W, int64_t ldw, const void* scale, void* C, int64_t ldc,
                      const void* R, int64_t ldr, int M, int N, int K, float alpha, cudaStream_t st);

}  // namespace npub

// Internal interface of the tcgen05 GEMM (gemm_tc.cu), shared with the
// attention host code.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstring>

namespace npub {

struct ZMap {
    int div, bat_hi, zrow_hi, zrow_lo;
};

struct GemmParams {
    CUtensorMap tmA;  // 128-row operand: box {64, 128, 1} or {64, 1, 128}; int8 raw or fp16 SW128
    CUtensorMap tmB;  // BT-row operand: fp16 SW128, box {64, BT, 1} or {64, 1, BT}
    int a_rows, b_rows, k_tiles;
    int a_row_dim, b_row_dim;  // tensor-map dimension (1 or 2) that indexes rows; the other indexes the batch
    // Batch index z (blockIdx.z / splits) is split as zl = z % zmod, zh = z / zmod; each operand maps it to
    // (batch coordinate, row offset) = (zl / div + zh * bat_hi, zh * zrow_hi + zl * zrow_lo).
    int zmod;
    ZMap za, zb;
    int splits, k_tiles_per_split;
    int causal_mode;           // 0 none; 1 skip tiles with b0 > a_last + off; 2 limit K to a_last + 1 + off
    int causal_off;
    void* out;
    int out_f32;               // 1: raw fp32 partials (split-K), no scale/residual
    int64_t o_sa, o_sb, o_split;  // output element strides: per A row, per B row, per split
    int64_t o_zl, o_zh;           // output offset per zl and per zh
    const __half* a_scale;     // per-A-row scale (output channel), may be null
    float alpha;
    const __half* res;         // residual, same indexing as the fp16 output, may be null
    int64_t r_sa, r_sb, r_zl, r_zh;
    int* err;                  // device error word
};

int num_sms();
int pick_bt(int b_rows);
// box0: elements of the innermost box dimension (64 = one 128-byte fp16 row;
// up to 256 for the unswizzled int8 weight tiles).
int make_tmap_3d(CUtensorMap* m, bool int8, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                 uint64_t s2, uint32_t box1, uint32_t box2, bool swizzle128, uint32_t box0 = 64);
int run_gemm(GemmParams& p, bool a_int8, int bt, int grid_x, int grid_y, int batch, cudaStream_t st);
// A plain (unbatched) mapping: zl = z, no row offsets.
inline void zmap_plain(GemmParams& p) {
    p.zmod = 1 << 30;
    p.za = ZMap{1, 0, 0, 0};
    p.zb = ZMap{1, 0, 0, 0};
}

}  // namespace npub

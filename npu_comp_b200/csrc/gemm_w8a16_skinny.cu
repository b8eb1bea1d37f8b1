// W8A16 GEMM for few tokens (M <= 64: decode steps), HBM-bound on the int8
// weight stream.
//
//   C[t, n] = fp16( alpha * scale[n] * sum_k A[t, k] * Wq[n, k] )  (+ R[t, n])
//
// D = Wq * A^T is computed in 128-row weight tiles (the MMA's M side) against
// all M tokens at once (the MMA's N side, BT = 32 or 64 columns).  The design
// follows from the weight stream being the whole cost:
//
//  * stream-K: the (tile, 256-wide K step) units are cut into one contiguous
//    range per CTA, grid = SM count, so every SM streams the same number of
//    weight bytes whatever N / 128 is.  A CTA walks its range in order, so a
//    tile cut between CTAs is the last tile of the CTA holding its first K
//    step (the tile's finisher) and the first tile of every other CTA holding
//    a piece of it.  Those other pieces are therefore done early: each stores
//    an fp32 partial and bumps the tile's counter (one per 32-row quarter, so
//    each epilogue warp works alone).  The finisher, at the end of its range,
//    waits for the counter, adds the partials to its own accumulator (read
//    straight from TMEM) in CTA order -- a fixed order, so results do not
//    depend on timing -- and stores the tile.  Only finishers wait, and only
//    on pieces that other CTAs compute first, so no wait can close a cycle;
//    grid <= SM count with one CTA per SM keeps every CTA resident.
//  * the converted weights never touch shared memory: converter warps read
//    the int8 tile (128-byte swizzled, conflict-free), turn it into fp16 in
//    registers and store it into tensor memory with tcgen05.st, where the
//    MMA reads it as the A operand (tcgen05.mma with A in TMEM).  Shared
//    memory carries only the TMA traffic.
//  * an int8 stage is released as soon as it is converted, not when the MMA
//    is done with it, so the int8 ring (2 x 32 KB) is all TMA in flight;
//    the token ring (L2-resident data, read by every CTA) is 3-4 deep.
//  * a K step is 256 wide: 16 MMAs per barrier wait and commit, which keeps
//    the single MMA thread's fixed per-step cost off the critical path.
//
// Roles (512 threads):
//   warp 0      TMA producer, int8 weights (ring of kS8 x 32 KB)
//   warp 1      TMEM allocator; MMA issuer
//   warp 2      TMA producer, fp16 tokens (ring of ST x BT x 128 x 2 B)
//   warps 4-7   epilogue: TMEM -> scale / residual -> fp16, or fp32 partials
//   warps 8-15  converters: every K step, warp 8 + 4h + q converts int8 box h
//               (bytes [128 h, 128 h + 128) of the step) of the rows of TMEM
//               lane quadrant q
//
// The tile counters fill the first kSkinnyCounterBytes of the workspace, the
// same bytes whatever the shape, so they are never overwritten by partials of
// another call.  They must be zero before the first call on a workspace and
// every completed call leaves them zero (the last piece of a tile resets its
// counter).
//
// Reference semantics: the NPU matmul (_poc/mysim.cpp:109-113,
// b_program_examples/npu.py:41-47) with float32 accumulation and an fp16 store.
#include "common.cuh"
#include "gemm_tc.h"
#include "gemm_w8a16_skinny.h"

#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <mutex>

namespace npub {

namespace skinny {

constexpr int kThreads = 512;
constexpr int kRows = 128;   // weight rows per tile (MMA M)
constexpr int kBK = 256;     // K per unit: two 128-byte swizzled int8 boxes per row, 16 MMAs per wait
constexpr int kBox8 = 128;   // int8 bytes of a row per TMA box (the 128-byte swizzle span)
constexpr int kS8 = 2;       // int8 ring depth (32 KB stages; 3 and 4 measured 0.3-0.7 % slower in decode)
constexpr int kSA = 3;       // fp16 weight stages in TMEM (kBK / 2 columns each)
constexpr int kPfUnits = 2;  // units of the next GEMM's CTAs prefetched to L2
constexpr int kRecvPad = 4;  // fp32 padding of each row of the cluster pieces in shared memory
constexpr int kConvWarps = 8;  // every converter warp works on every K step (half a row each)
constexpr int kAcols = kBK / 2;
constexpr int kAcol0 = 128;  // first TMEM column of the A stages (accumulators use [0, 2 BT) <= 128)
constexpr uint32_t kTmemCols = 512;
static_assert(kAcol0 + kSA * kAcols <= (int)kTmemCols, "tensor memory budget");

template <int BT>
struct Smem {
    static constexpr int kST = BT == 32 ? 4 : 3;  // token ring depth
    static constexpr int kTokChunk = BT * 128;    // 64 fp16 of K for BT tokens
    static constexpr int kTok = (kBK / 64) * kTokChunk;
    static constexpr int kA8Box = kRows * kBox8;
    static constexpr int kA8 = kRows * kBK;
    static constexpr int kRes = BT == 32 ? BT * kRows * 2 : 0;  // staged residual rows, fp16 [BT][kRows]
    static constexpr int kBars = 8 * (2 * kS8 + 2 * kST + 2 * kSA + 6) + 16 + 4 * BT;  // + row scales
    static constexpr int kTotal = kST * kTok + kS8 * kA8 + kRes + kBars + 1024;
};

// L2 (.cg) float4 store / load of the fp32 partials.  Volatile asm with a
// memory clobber: the loads of other CTAs' partials must stay behind the
// counter check and the fence that precede them (the compiler treats a
// plain asm load as free to move).
__device__ __forceinline__ void st_cg_f4(float4* ptr, float4 v) {
    asm volatile("st.global.cg.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(ptr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}
// 16-byte global -> shared copy that bypasses registers (the residual rows
// are staged while the accumulator is waited for).
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ float4 ld_cg_f4(const float4* ptr) {
    float4 v;
    asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(ptr)
                 : "memory");
    return v;
}

// Column sums of a warp's 32 x 16 block (lane = row): a butterfly that halves
// the columns each lane keeps at every step (16 shuffles).  Lanes 2c and
// 2c + 1 return the sum of column c' = 8 b4 + 4 b3 + 2 b2 + b1 (b = lane bits).
__device__ __forceinline__ float warp_colsum16(const float (&a)[16], int lane) {
    float b[8], c[4], d[2];
    const bool u4 = lane & 16, u3 = lane & 8, u2 = lane & 4, u1 = lane & 2;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float send = u4 ? a[k] : a[k + 8];
        b[k] = (u4 ? a[k + 8] : a[k]) + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float send = u3 ? b[k] : b[k + 4];
        c[k] = (u3 ? b[k + 4] : b[k]) + __shfl_xor_sync(0xffffffffu, send, 8);
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const float send = u2 ? c[k] : c[k + 2];
        d[k] = (u2 ? c[k + 2] : c[k]) + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    const float e = (u1 ? d[1] : d[0]) + __shfl_xor_sync(0xffffffffu, u1 ? d[0] : d[1], 2);
    return e + __shfl_xor_sync(0xffffffffu, e, 1);
}

__device__ __forceinline__ void epi_bar() { asm volatile("barrier.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ void set_err(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// Units [start(c), start(c+1)) belong to CTA c; owner(u) inverts that.
__device__ __forceinline__ int64_t unit_start(int64_t c, int64_t U, int64_t G) { return c * U / G; }
__device__ __forceinline__ int64_t unit_owner(int64_t u, int64_t U, int64_t G) { return ((u + 1) * G - 1) / U; }

// The segments of one CTA's unit range: one per tile it touches.
struct Range {
    int64_t u0, u1;
    int KT, tA, tB, nseg;
};

__device__ __forceinline__ Range make_range(int64_t u0, int64_t u1, int KT) {
    Range r;
    r.u0 = u0;
    r.u1 = u1;
    r.KT = KT;
    r.tA = (int)(u0 / KT);
    r.tB = (int)((u1 - 1) / KT);
    r.nseg = u1 > u0 ? r.tB - r.tA + 1 : 0;
    return r;
}

struct Seg {
    int tile, k0, nk;  // K steps [k0, k0 + nk) of the tile
    bool full;         // the whole tile: finished here, no partial
};

// i-th segment in processing order: the range's tiles in ascending order.
__device__ __forceinline__ Seg seg_in_order(const Range& r, int i) {
    const int t = r.tA + i;
    Seg s;
    s.tile = t;
    const int64_t ts = (int64_t)t * r.KT, te = ts + r.KT;
    const int64_t a = r.u0 > ts ? r.u0 : ts, b = r.u1 < te ? r.u1 : te;
    s.k0 = (int)(a - ts);
    s.nk = (int)(b - a);
    s.full = s.nk == r.KT;
    return s;
}

template <int BT>
__global__ void __launch_bounds__(kThreads, 1) w8a16_skinny_kernel(const __grid_constant__ SkinnyParams p) {
    pdl_trigger();
    using L = Smem<BT>;
    constexpr int kST = L::kST;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sTok = smem;                      // kST x kTok (1024-aligned)
    uint8_t* sA8 = sTok + kST * L::kTok;       // kS8 x kA8  (1024-aligned)
    __half* sRes = reinterpret_cast<__half*>(sA8 + kS8 * L::kA8);  // kRes: staged residual rows
    uint64_t* bars = reinterpret_cast<uint64_t*>(sA8 + kS8 * L::kA8 + L::kRes);
    uint64_t* full8 = bars;                    // [kS8] int8 tile landed
    uint64_t* empty8 = full8 + kS8;            // [kS8] int8 tile read by the 8 converter warps
    uint64_t* tok_full = empty8 + kS8;         // [kST] token tile landed
    uint64_t* tok_empty = tok_full + kST;      // [kST] MMA done with the token tile
    uint64_t* a_full = tok_empty + kST;        // [kSA] fp16 weights in TMEM (8 converter warps)
    uint64_t* a_empty = a_full + kSA;          // [kSA] MMA done with the TMEM stage
    uint64_t* acc_full = a_empty + kSA;        // [2] accumulator ready
    uint64_t* acc_empty = acc_full + 2;        // [2] epilogue drained the accumulator (4 warps)
    uint64_t* cl_go = acc_empty + 2;           // cluster split: the finisher's ring is free (1)
    uint64_t* cl_recv = cl_go + 1;             // cluster split: the other pieces are in (4 per piece)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(cl_recv + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* rstd_s = reinterpret_cast<float*>(tmem_slot + 4);  // [BT] row scales of a folded RMSNorm

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KT = p.k_steps;
    const int64_t U = (int64_t)p.n_tiles * KT, G = gridDim.x;
    // Cluster split (p.csplit = C > 1): cluster t computes tile t, its rank r
    // the K steps [r KT / C, (r + 1) KT / C); rank 0 finishes the tile from the
    // others' fp32 pieces, written into its idle int8 ring through distributed
    // shared memory.  Otherwise stream-K over the whole unit list.
    const int C = p.csplit > 1 ? p.csplit : 1;
    const uint32_t crank = C > 1 ? cluster_ctarank() : 0u;
    int64_t u0, u1;
    if (C > 1) {
        const int64_t t = blockIdx.x / C;
        u0 = t * KT + (int64_t)crank * KT / C;
        u1 = t * KT + (int64_t)(crank + 1) * KT / C;
    } else {
        u0 = unit_start(blockIdx.x, U, G);
        u1 = unit_start((int64_t)blockIdx.x + 1, U, G);
    }
    const Range rg = make_range(u0, u1, KT);
    // Cluster split with more than 16 tokens: converter warps 8-11 finish the
    // second 16-token block of the tile while epilogue warps 4-7 finish the
    // first (the epilogue's instruction latency, not its work, bounds it).
    const bool helpers = BT == 32 && C > 1 && p.M > 16;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kS8; ++s) {
            mbar_init(&full8[s], 1);
            mbar_init(&empty8[s], kConvWarps);
        }
        for (int s = 0; s < kST; ++s) {
            mbar_init(&tok_full[s], 1);
            mbar_init(&tok_empty[s], 1);
        }
        for (int s = 0; s < kSA; ++s) {
            mbar_init(&a_full[s], kConvWarps);
            mbar_init(&a_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        mbar_init(cl_go, 1);
        mbar_init(cl_recv, (helpers ? 8 : 4) * (C - 1));
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&p.tmW);
        prefetch_tmap(&p.tmX);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    cta_sync_divergent();
    tc_fence_after();
    if (C > 1) cluster_sync();  // every rank's barriers are initialised before any remote arrive
    bool cl_arrived = false;
    const uint32_t tmem = *tmem_slot;
    int never = 0;
    volatile int* no_abort = &never;
    // The weight producer, the converters and the MMA issuer touch only the
    // weights (never written by an earlier kernel), shared and tensor memory:
    // they start while the previous kernel finishes (measured: 1.7 % off a
    // batch-32 decode layer, 2 % off the stack's decode; holding the ring's
    // later stages back until the previous kernel is done costs 0.5-1.5 %,
    // while an extra L2 prefetch of the first tiles cost 0.3 %).  The token
    // producer and the epilogue (activations, residual, workspace) wait for it.
    if (warp == 0 || warp == 2) {
        // ------------------------------------------------------------ producers
        if (lane == 0) {
            const bool weights = warp == 0;
            if (!weights) pdl_wait();
            const uint64_t pol = l2_evict_first_policy();  // each weight is read once
            const int depth = weights ? kS8 : kST;
            uint64_t* full = weights ? full8 : tok_full;
            uint64_t* empty = weights ? empty8 : tok_empty;
            uint32_t g = 0;
            bool ok = true;
            for (int i = 0; i < rg.nseg && ok; ++i) {
                const Seg sg = seg_in_order(rg, i);
                for (int j = 0; j < sg.nk; ++j, ++g) {
                    const int k = (sg.k0 + j) * kBK;
                    const int s = (int)(g % (uint32_t)depth);
                    const uint32_t ph = (g / (uint32_t)depth) & 1u;
                    if (*abort_flag || !mbar_wait_bounded(&empty[s], ph ^ 1u, abort_flag)) {
                        *abort_flag = 1;
                        set_err(p.err, weights ? 0x301 : 0x302);
                        ok = false;
                        break;
                    }
                    if (weights) {
                        mbar_arrive_expect_tx(&full[s], (uint32_t)L::kA8);
#pragma unroll
                        for (int c = 0; c < kBK / kBox8; ++c) {
                            if (p.w_evict_first)
                                tma_load_3d_hint(sA8 + s * L::kA8 + c * L::kA8Box, &p.tmW, &full[s], k + c * kBox8,
                                                 sg.tile * kRows, 0, pol);
                            else
                                tma_load_3d(sA8 + s * L::kA8 + c * L::kA8Box, &p.tmW, &full[s], k + c * kBox8,
                                            sg.tile * kRows, 0);
                        }
                    } else {
                        mbar_arrive_expect_tx(&full[s], (uint32_t)L::kTok);
#pragma unroll
                        for (int c = 0; c < kBK / 64; ++c)
                            tma_load_3d(sTok + s * L::kTok + c * L::kTokChunk, &p.tmX, &full[s], k + 64 * c, 0, 0);
                    }
                }
            }
            if (weights && p.pf_grid > 0 && ok) {
                // this kernel's weights are all requested (it is MMA-bound, HBM has
                // room): the first units of the next GEMM's CTAs
                // [c G' / G, (c + 1) G' / G) go to L2 for its start
                prefetch_tmap(&p.tmWn);
                const int64_t G2 = p.pf_grid, KT2 = p.pf_ksteps, U2 = (int64_t)p.pf_tiles * KT2;
                const int cs = p.pf_csplit;
                for (int64_t c2 = (int64_t)blockIdx.x * G2 / G; c2 < ((int64_t)blockIdx.x + 1) * G2 / G; ++c2) {
                    int64_t a, e;
                    if (cs > 1) {
                        const int64_t t2 = c2 / cs, r2 = c2 % cs;
                        a = t2 * KT2 + r2 * KT2 / cs;
                        e = t2 * KT2 + (r2 + 1) * KT2 / cs;
                    } else {
                        a = unit_start(c2, U2, G2);
                        e = unit_start(c2 + 1, U2, G2);
                    }
                    for (int64_t u = a; u < e && u < a + kPfUnits; ++u)
#pragma unroll
                        for (int c = 0; c < kBK / kBox8; ++c)
                            tma_prefetch_3d(&p.tmWn, (int)(u % KT2) * kBK + c * kBox8, (int)(u / KT2) * kRows, 0);
                }
            }
            // Every load issued has landed before the CTA may exit.
            for (uint32_t j = 0; j < (uint32_t)depth && j < g; ++j) {
                const uint32_t gg = g - 1 - j;
                if (!mbar_wait_bounded(&full[gg % (uint32_t)depth], (gg / (uint32_t)depth) & 1u, no_abort,
                                       200000000ull))
                    set_err(p.err, 0x303);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(kRows, BT);
            uint32_t g = 0;
            bool ok = true;
            for (int t = 0; t < rg.nseg && ok; ++t) {
                const Seg sg = seg_in_order(rg, t);
                const uint32_t b = (uint32_t)t & 1u, bph = ((uint32_t)t >> 1) & 1u;
                if (!mbar_wait_bounded(&acc_empty[b], bph ^ 1u, abort_flag)) {
                    ok = false;
                    set_err(p.err, 0x304);
                    break;
                }
                tc_fence_after();
                const uint32_t dcol = tmem + b * (uint32_t)BT;
                for (int i = 0; i < sg.nk; ++i, ++g) {
                    const int sa = (int)(g % kSA), st = (int)(g % kST);
                    if (!mbar_wait_bounded(&a_full[sa], (g / kSA) & 1u, abort_flag) ||
                        !mbar_wait_bounded(&tok_full[st], (g / kST) & 1u, abort_flag)) {
                        ok = false;
                        set_err(p.err, 0x305);
                        break;
                    }
                    tc_fence_after();
                    const uint32_t acol = tmem + (uint32_t)(kAcol0 + sa * kAcols);
                    const uint32_t bbase = smem_u32(sTok + st * L::kTok);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {
                        const uint32_t baddr = bbase + (uint32_t)((kk >> 2) * L::kTokChunk + (kk & 3) * 32);
                        tc_mma_f16_ts(dcol, acol + (uint32_t)(kk * 8), umma_desc_sw128(baddr), idesc,
                                      (i > 0 || kk > 0) ? 1u : 0u);
                    }
                    tc_commit(&a_empty[sa]);
                    tc_commit(&tok_empty[st]);
                }
                if (!ok) break;
                tc_commit(&acc_full[b]);
            }
            if (!ok) *abort_flag = 1;
        }
    } else if (warp >= 8) {
        // ------------------------------------------------------------ converters
        const int half = (warp - 8) >> 2;  // which 64 bytes of K of the row
        const int q = warp & 3;            // TMEM lane quadrant of this warp
        const int row = 32 * q + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
        const int64_t total = rg.u1 - rg.u0;
        for (uint32_t g = 0; (int64_t)g < total; ++g) {
            const int s8 = (int)(g % kS8), sa = (int)(g % kSA);
            if (!mbar_wait_bounded(&full8[s8], (g / kS8) & 1u, abort_flag) ||
                !mbar_wait_bounded(&a_empty[sa], ((g / kSA) & 1u) ^ 1u, abort_flag)) {
                *abort_flag = 1;
                set_err(p.err, 0x306);
                break;
            }
            tc_fence_after();
            // this warp's half of the row: int8 box `half` (128 bytes, 128-byte swizzle)
            const uint8_t* src = sA8 + s8 * L::kA8 + half * L::kA8Box + row * kBox8;
            uint4 raw[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) raw[j] = *reinterpret_cast<const uint4*>(src + ((j ^ (row & 7)) << 4));
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty8[s8]);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t r[32];
#pragma unroll
                for (int j = 0; j < 4; ++j) i8x16_to_f16x2(raw[4 * h + j], &r[8 * j]);
                tmem_st32(lane_base + (uint32_t)(kAcol0 + sa * kAcols + 64 * half + 32 * h), r);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[sa]);
        }
    }
    if ((warp >= 4 && warp < 8) || (helpers && warp >= 8 && warp < 12)) {
        // ------------------------------------------------------------ epilogue
        pdl_wait();
        const bool helper = warp >= 8;
        // token blocks [c_lo, c_hi) of 16 that this warp finishes
        const int c_lo = helper ? 16 : 0, c_hi = helpers && !helper ? 16 : BT;
        const int q = warp & 3;
        const int r = 32 * q + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
        const int M = p.M;
        const SkinnyNorm& nm = p.nrm;
        if (nm.rs_part && !helper) {
            // row scales of the folded RMSNorm, while the first MMAs run: 128 / BT
            // threads per token sum its partials (8 loads in flight each) and
            // combine in a fixed order
            constexpr int P = 128 / BT;
            const int i = 32 * q + lane, tt = i / P, part = i % P;
            float s = 0.0f;
            if (tt < M) {
                const int lo = part * nm.rs_n / P, hi = (part + 1) * nm.rs_n / P;
                int k = lo;
                for (; k + 8 <= hi; k += 8) {
                    float x[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) x[u] = __ldcg(nm.rs_part + (int64_t)(k + u) * nm.rs_ld + tt);
#pragma unroll
                    for (int u = 0; u < 8; ++u) s += x[u];
                }
                for (; k < hi; ++k) s += __ldcg(nm.rs_part + (int64_t)k * nm.rs_ld + tt);
            }
#pragma unroll
            for (int o = 1; o < P; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (part == 0 && tt < BT) rstd_s[tt] = tt < M ? 1.0f / sqrtf(s / nm.rs_d + nm.rs_eps) : 0.0f;
            epi_bar();
        }
        if (nm.rs_part && helpers) {
            // the helpers read the row scales the epilogue warps wrote
            if (helper)
                asm volatile("barrier.sync 2, 256;" ::: "memory");
            else
                asm volatile("barrier.arrive 2, 256;" ::: "memory");
        }
        if ((p.R || nm.G) && !helper) {
            // the residual rows (and gamma) the stores will read go to L2 now,
            // while the MMAs run: read at the end, after the weight stream
            // has filled HBM's queues, they cost several microseconds
            for (int t = 0; t < rg.nseg; ++t) {
                const int n0 = seg_in_order(rg, t).tile * kRows + 32 * q;
                if (n0 >= p.N) continue;
                if (p.R && lane < M) asm volatile("prefetch.global.L2 [%0];" ::"l"(p.R + (int64_t)lane * p.ldr + n0));
                if (nm.G && lane == 0) asm volatile("prefetch.global.L2 [%0];" ::"l"(nm.gamma + n0));
            }
        }
        for (int t = 0; t < rg.nseg; ++t) {
            const Seg sg = seg_in_order(rg, t);
            const uint32_t b = (uint32_t)t & 1u, bph = ((uint32_t)t >> 1) & 1u;
            const int n = sg.tile * kRows + r;
            const bool nrow = n < p.N;
            // the scale and gamma loads and the residual rows' copy into shared
            // memory are in flight while the accumulator is waited for (read
            // in the epilogue, each was a dependent round trip of several
            // microseconds behind the memory traffic of the launch's end)
            const float sc = p.alpha * ((p.scale && nrow) ? __half2float(__ldg(p.scale + n)) : 1.0f);
            // (32-token tiles; the 64-token kernel has no registers to spare)
            constexpr bool kEarly = BT == 32;
            const float gm_early = (kEarly && nm.G && nrow) ? __half2float(__ldg(nm.gamma + n)) : 0.0f;
            if (kEarly && p.r_stage) {
                // this warp's 32 rows of the tile for every token: 64 bytes per token
                cp_async_wait_all();  // the previous segment's copy (same buffer) has landed
                __syncwarp();
                const int n0 = sg.tile * kRows + 32 * q;
                for (int id = 4 * c_lo + lane; id < 4 * min(M, c_hi); id += 32) {
                    const int tok = id >> 2, part = id & 3;
                    if (n0 + 8 * part < p.N)
                        cp_async16(sRes + tok * kRows + 32 * q + 8 * part, p.R + (int64_t)tok * p.ldr + n0 + 8 * part);
                }
                cp_async_commit();
            }
            bool res_ready = false;
            // The finished fp32 sums of this warp's 32 rows leave through
            // emit(): scaled (+ residual) and stored as fp16, or SwiGLU pairs.
            auto emit = [&](int c0, const float (&v)[16]) {
                float rs[16];  // row scales of a folded RMSNorm (1: none)
#pragma unroll
                for (int j = 0; j < 16; ++j) rs[j] = nm.rs_part ? rstd_s[c0 + j] : 1.0f;
                if (p.swiglu) {
                    // gate row 2c and up row 2c + 1 sit in adjacent lanes: both
                    // are rounded to fp16 as a separate GEMM would store them,
                    // and the pair forms fp16(silu(g) * u) for channel c
                    float gu[16], o[8];
#pragma unroll
                    for (int j = 0; j < 16; ++j) gu[j] = __half2float(__float2half_rn(v[j] * sc * rs[j]));
                    int t0;
                    swiglu_pair16(gu, lane, o, &t0);
                    if (!nrow) return;
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (c0 + t0 + j < M) p.C[(int64_t)(c0 + t0 + j) * p.ldc + n / 2] = __float2half_rn(o[j]);
                    return;
                }
                float rv[16];
                if (kEarly && p.r_stage) {
                    if (!res_ready) {
                        cp_async_wait_all();
                        __syncwarp();
                        res_ready = true;
                    }
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        rv[j] = (nrow && c0 + j < M) ? __half2float(sRes[(c0 + j) * kRows + r]) : 0.0f;
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        rv[j] = (p.R && nrow && c0 + j < M)
                                    ? __half2float(__ldg(p.R + (int64_t)(c0 + j) * p.ldr + n))
                                    : 0.0f;
                }
                __half o[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) o[j] = __float2half_rn(v[j] * sc * rs[j] + rv[j]);
                if (nm.ss) {
                    // the next RMSNorm's partial sums: this warp's 32 rows of C
                    float sq[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float f = __half2float(o[j]);
                        sq[j] = (nrow && c0 + j < M) ? f * f : 0.0f;
                    }
                    const float tot = warp_colsum16(sq, lane);
                    const int col = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
                    if (!(lane & 1) && c0 + col < M)
                        nm.ss[(int64_t)(sg.tile * 4 + q) * nm.ss_ld + c0 + col] = tot;
                }
                if (!nrow) return;
                const float gm = kEarly ? gm_early : (nm.G ? __half2float(__ldg(nm.gamma + n)) : 0.0f);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    if (c0 + j < M) {
                        p.C[(int64_t)(c0 + j) * p.ldc + n] = o[j];
                        if (nm.G) nm.G[(int64_t)(c0 + j) * nm.ldg + n] = __float2half_rn(__half2float(o[j]) * gm);
                    }
                }
            };
            if (C > 1) {
                // ---------------------------------------- cluster split: one segment per CTA
                bool have = mbar_wait_bounded(&acc_full[b], bph, abort_flag);
                if (!__all_sync(0xffffffffu, have)) {
                    if (lane == 0) set_err(p.err, 0x30a);
                    *abort_flag = 1;
                }
                tc_fence_after();
                // [C - 1][kRows][BT + 4] fp32 pieces (rank 0); the padded rows put the
                // 32 lanes' 16-byte accesses on different banks
                float* recv = reinterpret_cast<float*>(sA8);
                constexpr int RL = BT + kRecvPad;
                if (crank != 0) {
                    // wait until rank 0's MMAs are done (its ring is free), then write this
                    // piece into it and arrive on its barrier (release at cluster scope)
                    const bool go = __all_sync(0xffffffffu, mbar_wait_acq_cluster(cl_go, 0, abort_flag));
                    if (!go) {
                        if (lane == 0) set_err(p.err, 0x30b);
                        cluster_arrive();
                        cl_arrived = true;
                        continue;
                    }
                    const uint32_t dst =
                        mapa_shared(smem_u32(recv + ((int64_t)(crank - 1) * kRows + r) * RL), 0u);
                    for (int c0 = c_lo; c0 < c_hi && c0 < M; c0 += 16) {
                        float v[16];
                        tmem_ld16(lane_base + b * (uint32_t)BT + (uint32_t)c0, v);
#pragma unroll
                        for (int j = 0; j < 16; j += 4) st_cluster_f4(dst + 4u * (uint32_t)(c0 + j), v + j);
                    }
                    fence_acq_rel_cluster();  // every lane's stores before lane 0's release
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        if (!helper) mbar_arrive(&acc_empty[b]);
                        mbar_arrive_rel_cluster(mapa_shared(smem_u32(cl_recv), 0u));
                    }
                    cluster_arrive();  // this CTA's remote work is done
                    cl_arrived = true;
                    continue;
                }
                if (warp == 4 && lane == 0)
                    for (int rr = 1; rr < C; ++rr) mbar_arrive_rel_cluster(mapa_shared(smem_u32(cl_go), (uint32_t)rr));
                if (!mbar_wait_acq_cluster(cl_recv, 0, abort_flag) && lane == 0) set_err(p.err, 0x30c);
                cluster_arrive();  // every piece is in: the other ranks may leave
                cl_arrived = true;
                for (int c0 = c_lo; c0 < c_hi && c0 < M; c0 += 16) {
                    float v[16];
                    tmem_ld16(lane_base + b * (uint32_t)BT + (uint32_t)c0, v);
                    for (int rr = 1; rr < C; ++rr) {  // the pieces in rank order
                        const float4* pc = reinterpret_cast<const float4*>(recv + ((int64_t)(rr - 1) * kRows + r) * RL + c0);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float4 x = pc[j];
                            v[4 * j] += x.x;
                            v[4 * j + 1] += x.y;
                            v[4 * j + 2] += x.z;
                            v[4 * j + 3] += x.w;
                        }
                    }
                    emit(c0, v);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0 && !helper) mbar_arrive(&acc_empty[b]);
                continue;
            }
            // A tile cut between CTAs: its finisher is the CTA holding its first
            // K step; every other piece is the first tile of its CTA, whose one
            // partial slot it fills.
            int64_t c_first = blockIdx.x, c_last = blockIdx.x;
            if (!sg.full) {
                c_first = unit_owner((int64_t)sg.tile * KT, U, G);
                c_last = unit_owner((int64_t)sg.tile * KT + KT - 1, U, G);
            }
            const bool finisher = !sg.full && c_first == (int64_t)blockIdx.x;
            unsigned* cnt = p.cnt + 4 * sg.tile + q;
            // The finisher's epilogue warps wait for the other pieces while its
            // own MMAs run (they were computed first, so the wait is short) and
            // sum them in CTA order into S; the tile is own + S.
            float S[BT];
            if (finisher) {
                bool ok = true;
                if (lane == 0) {
                    const unsigned want = (unsigned)(c_last - c_first);
                    ok = ld_acquire_gpu(cnt) >= want;
                    if (!ok) {
                        const uint64_t t0 = globaltimer_ns();
                        for (uint32_t it = 1;; ++it) {
                            if (ld_acquire_gpu(cnt) >= want) {
                                ok = true;
                                break;
                            }
                            if ((it & 255u) == 0 && (*abort_flag || globaltimer_ns() - t0 > p.wait_ns)) break;
                        }
                    }
                    if (ok) *cnt = 0u;  // left zero for the next call
                }
                ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
                if (!ok) {
                    set_err(p.err, 0x309);
                    *abort_flag = 1;
                    break;
                }
                __threadfence();
                {
                    // the first later piece straight into S, all loads in flight
                    const float4* pp = reinterpret_cast<const float4*>(p.part + ((c_first + 1) * kRows + r) * BT);
#pragma unroll
                    for (int c0 = 0; c0 < BT; c0 += 16) {
                        if (c0 < M) {
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const float4 x = ld_cg_f4(pp + c0 / 4 + j);
                                S[c0 + 4 * j] = x.x;
                                S[c0 + 4 * j + 1] = x.y;
                                S[c0 + 4 * j + 2] = x.z;
                                S[c0 + 4 * j + 3] = x.w;
                            }
                        }
                    }
                }
                for (int64_t c = c_first + 2; c <= c_last; ++c) {
                    const float4* pp = reinterpret_cast<const float4*>(p.part + (c * kRows + r) * BT);
#pragma unroll
                    for (int c0 = 0; c0 < BT; c0 += 16) {
                        if (c0 < M) {
                            float4 x[4];
#pragma unroll
                            for (int j = 0; j < 4; ++j) x[j] = ld_cg_f4(pp + c0 / 4 + j);
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                S[c0 + 4 * j] += x[j].x;
                                S[c0 + 4 * j + 1] += x[j].y;
                                S[c0 + 4 * j + 2] += x[j].z;
                                S[c0 + 4 * j + 3] += x[j].w;
                            }
                        }
                    }
                }
            }
            bool have = mbar_wait_bounded(&acc_full[b], bph, abort_flag);
            if (!have) set_err(p.err, 0x307);
            have = __all_sync(0xffffffffu, have);
            if (!have) {
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            if (sg.full) {
                for (int c0 = 0; c0 < BT && c0 < M; c0 += 16) {
                    float v[16];
                    tmem_ld16(lane_base + b * (uint32_t)BT + (uint32_t)c0, v);
                    emit(c0, v);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[b]);
                continue;
            }
            if (!finisher) {
                // a later piece: fp32 partial [slot = CTA][row][BT], then publish it
                float4* mine = reinterpret_cast<float4*>(p.part + ((int64_t)blockIdx.x * kRows + r) * BT);
                for (int c0 = 0; c0 < BT && c0 < M; c0 += 16) {
                    float v[16];
                    tmem_ld16(lane_base + b * (uint32_t)BT + (uint32_t)c0, v);
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        st_cg_f4(mine + c0 / 4 + j, make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[b]);
                __threadfence();
                __syncwarp();
                if (lane == 0) atomicAdd(cnt, 1u);
                continue;
            }
            // the finisher: own accumulator + S, scaled and stored
#pragma unroll
            for (int c0 = 0; c0 < BT; c0 += 16) {
                if (c0 < M) {
                    float v[16];
                    tmem_ld16(lane_base + b * (uint32_t)BT + (uint32_t)c0, v);
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] += S[c0 + j];
                    emit(c0, v);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
        if (BT == 32 && p.r_stage) cp_async_wait_all();  // no copy into shared memory outlives the CTA
    }

    // Lane 0 alone ran some warps' role loops: a thread-counting barrier.
    // Cluster split: no CTA leaves before every CTA of its cluster has arrived
    // (after its last access to another CTA's shared memory).
    if (C > 1 && !cl_arrived) cluster_arrive();
    tc_fence_before();
    cta_sync_divergent();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    if (C > 1) cluster_wait();
}

template <int BT>
static int launch(const SkinnyParams& p, int grid, cudaStream_t st) {
    using L = Smem<BT>;
    static_assert(L::kTotal <= 232448, "shared memory budget");
    auto kern = w8a16_skinny_kernel<BT>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
    if (e != cudaSuccess) {
        npub_internal_set_cuda_error(e);
        return NPUB_ERR_CUDA;
    }
    if (p.csplit <= 1) return launch_pdl(kern, dim3(grid), dim3(kThreads), L::kTotal, st, p);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L::kTotal;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = npub_internal_pdl_enabled() ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)p.csplit;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) {
        npub_internal_set_cuda_error(e);
        return NPUB_ERR_CUDA;
    }
    return npub_internal_launch_status();
}

// Clusters of c stream-K kernels that can be resident at once (0: none).
template <int BT>
static int max_clusters(int c) {
    using L = Smem<BT>;
    auto kern = w8a16_skinny_kernel<BT>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c * 64);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L::kTotal;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = (unsigned)c;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

}  // namespace skinny

int skinny_bt(int M) { return M <= 32 ? 32 : 64; }

// One CTA per SM, but at least a quarter of a tile's K steps per CTA: a tile
// is cut into at most ~5 pieces, which bounds the fixup of small matrices.
static int skinny_grid(int N, int K) {
    const int64_t kt = (K + skinny::kBK - 1) / skinny::kBK;
    const int64_t units = (int64_t)((N + skinny::kRows - 1) / skinny::kRows) * kt;
    const int64_t min_units = (kt + 3) / 4;
    const int64_t want = (units + min_units - 1) / min_units;
    const int sms = num_sms();
    return (int)(want < sms ? want : sms);
}

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Cluster split for matrices of few 128-row tiles (the decode step's O and
// down projections at d = 4096: 32 tiles): C = SMs / tiles CTAs per tile
// (2..8) when they fill most of the GPU, every cluster can be resident at
// once and each piece has at least two K steps.  The pieces then meet in the
// finisher's shared memory instead of global memory (the stream-K partials'
// store / fence / counter / load chain cost ~5 us per launch behind the
// weight stream).  NPUB_SKINNY_CLUSTER=0 in the environment keeps stream-K.
static int skinny_csplit(int bt, int n_tiles, int k_steps) {
    static const bool off = [] {
        const char* e = getenv("NPUB_SKINNY_CLUSTER");
        return e && e[0] == '0';
    }();
    const int sms = num_sms();
    if (off || n_tiles <= 0) return 1;
    const int c = std::min(8, sms / n_tiles);
    if (c < 2 || n_tiles * c * 5 < sms * 4 || k_steps < 2 * c) return 1;
    // the other pieces land in the finisher's int8 ring
    if ((size_t)(c - 1) * skinny::kRows * (bt + skinny::kRecvPad) * sizeof(float) >
        (size_t)skinny::kS8 * skinny::kRows * skinny::kBK)
        return 1;
    static std::mutex mu;
    static int cache[2][9];
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    int& mc = cache[bt == 32 ? 0 : 1][c];
    if (mc == 0) mc = 1 + (bt == 32 ? skinny::max_clusters<32>(c) : skinny::max_clusters<64>(c));
    return mc - 1 >= n_tiles ? c : 1;
}

bool w8a16_skinny_fits(int M, int N) {
    return M > 0 && M <= kSkinnyMaxM && N > 0 &&
           (size_t)4 * ((N + skinny::kRows - 1) / skinny::kRows) * sizeof(unsigned) <= kSkinnyCounterBytes;
}

// Measured on B200 (decode-layer shapes, weights streamed from HBM, CUDA
// graph replay): the stream-K kernel wins on every matrix with N >= 8192 and,
// at M <= 32, on K-long ones (4096 x 11008) and, inside a decode layer, on
// the square 4096 x 4096 projection (215.6 vs 219.0 us per batch-32 layer:
// its weights stream while the attention kernel finishes, although alone it
// is slower, 22.9 vs 21.7 us); the 2-CTA pair kernel wins on the square and
// K-long ones at M = 64 (745 vs 754 us per batch-64 layer), where its wider
// MMAs issue fewer instructions per weight byte.
// NPUB_W8A16_KERNEL=pair or =skinny in the environment overrides the choice
// (where the shape allows it), for measuring both kernels on one shape.
static int kernel_override() {
    static const int v = [] {
        const char* e = getenv("NPUB_W8A16_KERNEL");
        if (!e) return 0;
        if (!strcmp(e, "pair")) return 1;
        if (!strcmp(e, "skinny")) return 2;
        return 0;
    }();
    return v;
}

bool w8a16_use_skinny(int M, int N, int K) {
    if (!w8a16_skinny_fits(M, N) || K <= 0) return false;
    const int o = kernel_override();
    if (o) return o == 2;
    return N >= 8192 || (M <= 32 && (K >= 8192 || (N >= 4096 && K >= 4096)));
}

size_t w8a16_skinny_workspace(int M, int N, int K) {
    if (!w8a16_skinny_fits(M, N) || K <= 0) return 0;
    return kSkinnyCounterBytes + (size_t)skinny_grid(N, K) * skinny_bt(M) * skinny::kRows * sizeof(float);
}

int w8a16_skinny_run(const void* A, int64_t lda, const void* W, int64_t ldw, const void* scale, void* C, int64_t ldc,
                     const void* R, int64_t ldr, int M, int N, int K, float alpha, void* ws, size_t ws_bytes,
                     cudaStream_t st, int swiglu, const SkinnyNorm* nrm, const SkinnyNext* next) {
    if (!w8a16_skinny_fits(M, N)) return NPUB_ERR_INVALID_ARG;
    if (swiglu && (N % 2 || R)) return NPUB_ERR_INVALID_ARG;
    const size_t need = w8a16_skinny_workspace(M, N, K);
    if (!ws || ws_bytes < need) return NPUB_ERR_WORKSPACE;
    if (!npub_aligned(ws, 16)) return NPUB_ERR_INVALID_ARG;
    const int bt = skinny_bt(M);
    SkinnyParams p;
    memset(&p, 0, sizeof(p));
    int rc = make_tmap_3d(&p.tmW, true, W, (uint64_t)K, (uint64_t)N, 1, (uint64_t)ldw, (uint64_t)ldw * N,
                          skinny::kRows, 1, true, skinny::kBox8);
    if (rc) return rc;
    rc = make_tmap_3d(&p.tmX, false, A, (uint64_t)K, (uint64_t)M, 1, (uint64_t)lda, (uint64_t)lda * M, (uint32_t)bt,
                      1, true);
    if (rc) return rc;
    p.M = M;
    p.N = N;
    p.w_evict_first = npub_internal_l2_evict_first() ? 1 : 0;
    p.k_steps = (K + skinny::kBK - 1) / skinny::kBK;
    p.n_tiles = (N + skinny::kRows - 1) / skinny::kRows;
    p.C = reinterpret_cast<__half*>(C);
    p.ldc = ldc;
    p.R = reinterpret_cast<const __half*>(R);
    p.ldr = ldr;
    static const bool r_stage_off = [] {
        const char* e = getenv("NPUB_SKINNY_RSTAGE");
        return e && e[0] == '0';
    }();
    p.r_stage = (R && !r_stage_off && npub_aligned(R, 16) && ldr % 8 == 0 && N % 8 == 0) ? 1 : 0;
    p.scale = reinterpret_cast<const __half*>(scale);
    p.alpha = alpha;
    p.cnt = reinterpret_cast<unsigned*>(ws);
    p.part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + kSkinnyCounterBytes);
    p.err = npub_internal_device_error_word();
    p.wait_ns = npub_internal_wait_limit_ns();
    p.swiglu = swiglu ? 1 : 0;
    if (nrm) p.nrm = *nrm;
    p.csplit = skinny_csplit(bt, p.n_tiles, p.k_steps);
    const int grid = p.csplit > 1 ? p.n_tiles * p.csplit : skinny_grid(N, K);
    if (next && next->W && w8a16_skinny_fits(next->M, next->N) && next->K > 0 && next->K % 16 == 0 &&
        next->ldw >= next->K && next->ldw % 16 == 0 && npub_aligned(next->W, 16)) {
        rc = make_tmap_3d(&p.tmWn, true, next->W, (uint64_t)next->K, (uint64_t)next->N, 1, (uint64_t)next->ldw,
                          (uint64_t)next->ldw * next->N, skinny::kRows, 1, true, skinny::kBox8);
        if (rc) return rc;
        p.pf_tiles = (next->N + skinny::kRows - 1) / skinny::kRows;
        p.pf_ksteps = (next->K + skinny::kBK - 1) / skinny::kBK;
        p.pf_csplit = skinny_csplit(skinny_bt(next->M), p.pf_tiles, p.pf_ksteps);
        p.pf_grid = p.pf_csplit > 1 ? p.pf_tiles * p.pf_csplit : skinny_grid(next->N, next->K);
    }
    return bt == 32 ? skinny::launch<32>(p, grid, st) : skinny::launch<64>(p, grid, st);
}

}  // namespace npub

// W8A16 GEMM for prefill-sized M on 2-CTA tensor-core pairs, with the
// converted fp16 weights in tensor memory.
//
//   C[t, n] = fp16( alpha * scale[n] * sum_k A[t, k] * Wq[n, k] )  (+ R[t, n])
//
// A cluster of two CTAs computes a 256 x 192 tile of D = Wq * A^T with
// tcgen05.mma.cta_group::2 (M = 256 weight rows, N = 192 tokens).  CTA r of
// the pair owns weight rows [a0 + 128 r, a0 + 128 r + 128) and loads token rows
// [b0 + 96 r, b0 + 96 r + 96) (its half of the N side).
//
// Why tensor memory: converting the int8 weights into shared memory, as an
// fp16 GEMM would hold them, costs two 16-byte shared stores per 16 weights and
// a second read of the same bytes by the tensor core; with a 256-token tile
// those shared-memory wavefronts take half of the LSU budget of the
// shared-memory pair kernel (gemm_w8a16_pair.cu).  Here converter warps turn each int8 row
// slice into fp16 pairs in registers and store it with tcgen05.st into the
// CTA's tensor memory, and the MMA reads A from there ([a-tmem] form).  Shared
// memory carries only the TMA traffic (int8 weights, fp16 tokens) and the B
// operand reads.
//
// Tensor memory per CTA (512 columns): two 192-column fp32 accumulators
// (the epilogue of one tile overlaps the main loop of the next) and four
// 32-column fp16 weight stages of 64 K each.
//
// Roles per CTA (512 threads):
//   warp 0      TMA producer, int8 weights (ring of kS8 x 16 KB, 128-byte swizzle)
//   warp 1      TMEM allocator (both CTAs); MMA issuer (even CTA)
//   warp 2      TMA producer, token half-tiles -> the even CTA's barrier
//   warps 4-7   epilogue: TMEM -> scale / residual -> fp16
//   warps 8-15  converters: warp 8 + 4h + q converts K half h of every int8
//               stage for the rows of TMEM lane quadrant q
// No TMA load uses multicast.  Every wait is bounded and sets an error code.
//
// Reference semantics: the NPU matmul (_poc/mysim.cpp:109-113,
// b_program_examples/npu.py:41-47) with float32 accumulation and an fp16 store.
#include "common.cuh"
#include "gemm_tc.h"
#include "gemm_w8a16_pair_ts.h"

#include <cstdlib>
#include <cstring>
#include <mutex>

namespace npub {

namespace pts {

constexpr int kThreads = 512;
constexpr int kRows = 128;         // weight rows per CTA
constexpr int kBT = 192;           // tokens per tile (MMA N)
constexpr int kHalfBT = kBT / 2;   // token rows per CTA
constexpr int kBK = 128;           // K per TMA stage: one 128-byte swizzled int8 row
constexpr int kS8 = 6;             // int8 ring depth (16 KB stages)
constexpr int kST = 4;             // token ring depth (24 KB stages)
constexpr int kSA = 4;             // fp16 weight stages in TMEM (64 K each)
constexpr int kAcols = 32;         // TMEM columns of one weight stage
constexpr int kAcol0 = 2 * kBT;    // accumulators use columns [0, 2 kBT)
constexpr uint32_t kTmemCols = 512;
static_assert(kAcol0 + kSA * kAcols <= (int)kTmemCols, "tensor memory budget");
static_assert(kSA % 2 == 0, "one int8 stage fills two weight stages");

struct Smem {
    static constexpr int kA8 = kRows * kBK;              // 16 KB
    static constexpr int kTokChunk = kHalfBT * 128;       // 64 fp16 of K for 96 token rows
    static constexpr int kTok = (kBK / 64) * kTokChunk;   // 24 KB
    static constexpr int kBars = 8 * (2 * kS8 + 2 * kST + 2 * kSA + 4) + 16;
    static constexpr int kTotal = kST * kTok + kS8 * kA8 + kBars + 1024;
};

__device__ __forceinline__ void set_err(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// Tile order: bands of up to kBand token tiles; within a band the weight pairs
// in turn, each against every token tile of the band.  The ~74 tiles in
// flight then share a few weight pairs and one band of tokens, so both stay
// in L2: tokens come from HBM once, weights once per band.
constexpr int kBand = 12;
__device__ __forceinline__ void tile_ab(const PairTsParams& p, int tile, int& ap, int& bi) {
    const int per_band = kBand * p.n_apairs;
    const int band = tile / per_band;
    const int r = tile - band * per_band;
    const int nb = min(kBand, p.n_btiles - band * kBand);  // token tiles in this band
    ap = r / nb;
    bi = band * kBand + r % nb;
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    w8a16_pair_ts_kernel(const __grid_constant__ PairTsParams p) {
    pdl_trigger();
    using L = Smem;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sTok = smem;                  // kST x kTok (1024-aligned)
    uint8_t* sA8 = sTok + kST * L::kTok;   // kS8 x kA8  (1024-aligned)
    uint64_t* bars = reinterpret_cast<uint64_t*>(sA8 + kS8 * L::kA8);
    uint64_t* full8 = bars;                // [kS8] int8 tile landed (own)
    uint64_t* empty8 = full8 + kS8;        // [kS8] int8 tile read by the 8 converter warps (own)
    uint64_t* tok_full = empty8 + kS8;     // [kST] (even CTA) both token halves landed
    uint64_t* tok_empty = tok_full + kST;  // [kST] pair MMA done with the token stage
    uint64_t* a_full = tok_empty + kST;    // [kSA] (even CTA) both CTAs' weight stage in TMEM
    uint64_t* a_empty = a_full + kSA;      // [kSA] pair MMA done with the weight stage
    uint64_t* acc_full = a_empty + kSA;    // [2] accumulator ready
    uint64_t* acc_empty = acc_full + 2;    // [2] (even CTA) both epilogues drained the buffer
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int cid = (int)cluster_id_x(), ncl = (int)nclusters_x();
    const int KT = p.k_steps;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kS8; ++s) {
            mbar_init(&full8[s], 1);
            mbar_init(&empty8[s], 8);
        }
        for (int s = 0; s < kST; ++s) {
            mbar_init(&tok_full[s], 1);
            mbar_init(&tok_empty[s], 1);
        }
        for (int s = 0; s < kSA; ++s) {
            mbar_init(&a_full[s], 8);  // 2 CTAs x 4 converter warps
            mbar_init(&a_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 8);  // 2 CTAs x 4 epilogue warps
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&p.tmW);
        prefetch_tmap(&p.tmX);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // barriers of both CTAs initialised before any remote arrive
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    int never = 0;
    volatile int* no_abort = &never;
    pdl_wait();

    if (warp == 0) {
        // ------------------------------------------------------------ int8 weights
        if (lane == 0) {
            uint32_t g = 0;
            bool ok = true;
            for (int tile = cid; tile < p.n_tiles && ok; tile += ncl) {
                int ap, bi;
                tile_ab(p, tile, ap, bi);
                const int arow = ap * 2 * kRows + (int)rank * kRows;
                for (int i = 0; i < KT; ++i, ++g) {
                    const int s = (int)(g % kS8);
                    if (*abort_flag || !mbar_wait_bounded(&empty8[s], ((g / kS8) & 1u) ^ 1u, abort_flag)) {
                        *abort_flag = 1;
                        set_err(p.err, 0x601);
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full8[s], (uint32_t)L::kA8);
                    tma_load_3d(sA8 + s * L::kA8, &p.tmW, &full8[s], i * kBK, arow, 0);
                }
            }
            // every load issued has landed before the CTA may exit
            for (uint32_t j = 0; j < (uint32_t)kS8 && j < g; ++j) {
                const uint32_t gg = g - 1 - j;
                if (!mbar_wait_bounded(&full8[gg % kS8], (gg / kS8) & 1u, no_abort, 200000000ull))
                    set_err(p.err, 0x602);
            }
        }
    } else if (warp == 2) {
        // ------------------------------------------------------------ token half-tiles
        if (lane == 0) {
            const uint32_t tok_full0 = mapa_shared(smem_u32(&tok_full[0]), 0);
            uint32_t g = 0;
            bool ok = true;
            for (int tile = cid; tile < p.n_tiles && ok; tile += ncl) {
                int ap, bi;
                tile_ab(p, tile, ap, bi);
                const int brow = bi * kBT + (int)rank * kHalfBT;
                for (int i = 0; i < KT; ++i, ++g) {
                    const int s = (int)(g % kST);
                    if (*abort_flag ||
                        !mbar_wait_cluster_bounded(&tok_empty[s], ((g / kST) & 1u) ^ 1u, abort_flag)) {
                        *abort_flag = 1;
                        set_err(p.err, 0x603);
                        ok = false;
                        break;
                    }
                    if (leader) mbar_arrive_expect_tx(&tok_full[s], (uint32_t)(2 * L::kTok));
#pragma unroll
                    for (int ch = 0; ch < kBK / 64; ++ch)
                        tma_load_3d_pair(sTok + s * L::kTok + ch * L::kTokChunk, &p.tmX, tok_full0 + (uint32_t)s * 8u,
                                         i * kBK + 64 * ch, brow, 0);
                }
            }
            // Both CTAs' token loads signal the even CTA's barriers: it waits for
            // the last ones (already consumed unless the MMA issuer gave up),
            // and the final cluster barrier keeps the odd CTA until then.
            if (leader)
                for (uint32_t j = 0; j < (uint32_t)kST && j < g; ++j) {
                    const uint32_t gg = g - 1 - j;
                    if (!mbar_wait_cluster_bounded(&tok_full[gg % kST], (gg / kST) & 1u, no_abort, 200000000ull))
                        set_err(p.err, 0x609);
                }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (leader && lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(2 * kRows, kBT);
            const uint32_t peer = 1u;
            uint32_t gt = 0, ga = 0, t = 0;
            bool ok = true;
            for (int tile = cid; tile < p.n_tiles && ok; tile += ncl, ++t) {
                const uint32_t b = t & 1u, bph = (t >> 1) & 1u;
                if (!mbar_wait_cluster_bounded(&acc_empty[b], bph ^ 1u, abort_flag)) {
                    ok = false;
                    set_err(p.err, 0x604);
                    break;
                }
                tc_fence_after();
                const uint32_t dcol = tmem + b * (uint32_t)kBT;
                for (int i = 0; i < KT && ok; ++i, ++gt) {
                    const int st = (int)(gt % kST);
                    if (!mbar_wait_cluster_bounded(&tok_full[st], (gt / kST) & 1u, abort_flag)) {
                        ok = false;
                        set_err(p.err, 0x605);
                        break;
                    }
#pragma unroll
                    for (int h = 0; h < kBK / 64; ++h, ++ga) {
                        const int sa = (int)(ga % kSA);
                        if (!mbar_wait_cluster_bounded(&a_full[sa], (ga / kSA) & 1u, abort_flag)) {
                            ok = false;
                            set_err(p.err, 0x606);
                            break;
                        }
                        tc_fence_after();
                        const uint32_t acol = tmem + (uint32_t)(kAcol0 + sa * kAcols);
                        const uint32_t bbase = smem_u32(sTok + st * L::kTok + h * L::kTokChunk);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            tc_mma_f16_pair_ts(dcol, acol + (uint32_t)(kk * 8), umma_desc_sw128(bbase + kk * 32),
                                               idesc, (i > 0 || h > 0 || kk > 0) ? 1u : 0u);
                        tc_commit_pair(smem_u32(&a_empty[sa]));
                        tc_commit_pair(mapa_shared(smem_u32(&a_empty[sa]), peer));
                    }
                    if (!ok) break;
                    tc_commit_pair(smem_u32(&tok_empty[st]));
                    tc_commit_pair(mapa_shared(smem_u32(&tok_empty[st]), peer));
                }
                if (!ok) break;
                tc_commit_pair(smem_u32(&acc_full[b]));
                tc_commit_pair(mapa_shared(smem_u32(&acc_full[b]), peer));
            }
            if (!ok) *abort_flag = 1;
        }
    } else if (warp >= 8) {
        // ------------------------------------------------------------ converters
        const int h = (warp - 8) >> 2;  // which 64 bytes of K of the row
        const int q = warp & 3;         // TMEM lane quadrant of this warp
        const int row = 32 * q + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
        const uint32_t a_full0 = mapa_shared(smem_u32(&a_full[0]), 0);
        uint32_t g = 0;
        bool ok = true;
        for (int tile = cid; tile < p.n_tiles && ok; tile += ncl) {
            for (int i = 0; i < KT; ++i, ++g) {
                const int s8 = (int)(g % kS8);
                const uint32_t ga = 2u * g + (uint32_t)h;
                const int sa = (int)(ga % kSA);
                if (!mbar_wait_bounded(&full8[s8], (g / kS8) & 1u, abort_flag) ||
                    !mbar_wait_cluster_bounded(&a_empty[sa], ((ga / kSA) & 1u) ^ 1u, abort_flag)) {
                    *abort_flag = 1;
                    set_err(p.err, 0x607);
                    ok = false;
                    break;
                }
                tc_fence_after();
                // this warp's half of the row: 16-byte chunks 4h .. 4h + 3 (128-byte swizzle)
                const uint8_t* src = sA8 + s8 * L::kA8 + row * kBK;
                uint4 raw[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) raw[j] = *reinterpret_cast<const uint4*>(src + (((4 * h + j) ^ (row & 7)) << 4));
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty8[s8]);
                uint32_t r[32];
#pragma unroll
                for (int j = 0; j < 4; ++j) i8x16_to_f16x2(raw[j], &r[8 * j]);
                tmem_st32(lane_base + (uint32_t)(kAcol0 + sa * kAcols), r);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(a_full0 + (uint32_t)sa * 8u);
            }
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------ epilogue
        const int wq = warp & 3;
        const uint32_t acc_empty0 = mapa_shared(smem_u32(&acc_empty[0]), 0);
        uint32_t t = 0;
        for (int tile = cid; tile < p.n_tiles; tile += ncl, ++t) {
            int ap, bi;
            tile_ab(p, tile, ap, bi);
            const int a0 = ap * 2 * kRows, b0 = bi * kBT;
            const uint32_t b = t & 1u, bph = (t >> 1) & 1u;
            const int n = a0 + (int)rank * kRows + wq * 32 + lane;
            const bool nrow = n < p.N;
            // the scale load is in flight while the accumulator is waited for
            const float sc = p.alpha * ((p.scale && nrow) ? __half2float(__ldg(p.scale + n)) : 1.0f);
            bool have = mbar_wait_cluster_bounded(&acc_full[b], bph, abort_flag);
            if (!have) set_err(p.err, 0x608);
            have = __all_sync(0xffffffffu, have);
            if (!have) {
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            for (int c0 = 0; c0 < kBT; c0 += 16) {
                if (b0 + c0 >= p.M) break;  // warp-uniform
                float v[16];
                tmem_ld16(tmem + ((uint32_t)(wq * 32) << 16) + b * (uint32_t)kBT + (uint32_t)c0, v);
                if (!nrow) continue;
                const int tb = b0 + c0;
                // all residual loads are issued before the first store
                float rv[16];
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    rv[j] = (p.R && tb + j < p.M) ? __half2float(__ldg(p.R + (int64_t)(tb + j) * p.ldr + n)) : 0.0f;
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (tb + j < p.M) p.C[(int64_t)(tb + j) * p.ldc + n] = __float2half_rn(v[j] * sc + rv[j]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc_empty0 + b * 8u);
        }
    }

    // Lane 0 alone ran some warps' role loops: thread-counting barriers.
    tc_fence_before();
    cta_sync_divergent();
    cluster_sync();  // no CTA leaves while its peer may still signal or read it
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, kTmemCols);
    }
}

static std::mutex g_mu;
static int g_max_clusters[64];

static int max_clusters(int dev) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_max_clusters[dev] > 0) return g_max_clusters[dev];
    auto kern = w8a16_pair_ts_kernel;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem::kTotal);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 256, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = Smem::kTotal;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = num_sms() / 2;
    }
    g_max_clusters[dev] = n;
    return n;
}

}  // namespace pts

// Measured on B200 (2048 x 22016 x 4096, L2 flushed): 878-910 TFLOP/s against
// 1060-1150 for the shared-memory pair kernel.  The shared-memory traffic it
// was built to remove is gone (ncu: LSU shared wavefronts 9.7 % vs 50.4 %),
// but its tensor pipe is busier per FLOP: in-kernel timers give ~121 SM cycles
// per N = 192 MMA against 96 for the same instruction stream in isolation
// (converter TMEM stores, epilogue TMEM loads, commits, fences and concurrent
// shared-memory writes each measured not to matter), and the issuing thread
// is busy ~72 % of the time.  It is therefore opt-in: NPUB_W8A16_KERNEL=pair_ts
// in the environment selects it for every shape it supports (M > 64).
static int pair_ts_override() {
    static const int v = [] {
        const char* e = getenv("NPUB_W8A16_KERNEL");
        return (e && !strcmp(e, "pair_ts")) ? 1 : 0;
    }();
    return v;
}

bool w8a16_use_pair_ts(int M, int N, int K) {
    if (M <= 64 || N <= 0 || K <= 0) return false;
    return pair_ts_override() == 1;
}

int w8a16_pair_ts_run(const void* A, int64_t lda, const void* W, int64_t ldw, const void* scale, void* C, int64_t ldc,
                      const void* R, int64_t ldr, int M, int N, int K, float alpha, cudaStream_t st) {
    PairTsParams p;
    memset(&p, 0, sizeof(p));
    int rc = make_tmap_3d(&p.tmW, true, W, (uint64_t)K, (uint64_t)N, 1, (uint64_t)ldw, (uint64_t)ldw * N, pts::kRows, 1,
                          true, pts::kBK);
    if (rc) return rc;
    rc = make_tmap_3d(&p.tmX, false, A, (uint64_t)K, (uint64_t)M, 1, (uint64_t)lda, (uint64_t)lda * M,
                      (uint32_t)pts::kHalfBT, 1, true);
    if (rc) return rc;
    p.M = M;
    p.N = N;
    p.k_steps = (K + pts::kBK - 1) / pts::kBK;
    p.n_apairs = (N + 2 * pts::kRows - 1) / (2 * pts::kRows);
    p.n_btiles = (M + pts::kBT - 1) / pts::kBT;
    p.n_tiles = p.n_apairs * p.n_btiles;
    p.C = reinterpret_cast<__half*>(C);
    p.ldc = ldc;
    p.R = reinterpret_cast<const __half*>(R);
    p.ldr = ldr;
    p.scale = reinterpret_cast<const __half*>(scale);
    p.alpha = alpha;
    p.err = npub_internal_device_error_word();
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
    int clusters = pts::max_clusters(dev);
    if (clusters > p.n_tiles) clusters = p.n_tiles;
    if (clusters < 1) clusters = 1;
    cudaError_t e = cudaFuncSetAttribute(pts::w8a16_pair_ts_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         pts::Smem::kTotal);
    if (e != cudaSuccess) {
        npub_internal_set_cuda_error(e);
        return NPUB_ERR_CUDA;
    }
    static_assert(pts::Smem::kTotal <= 232448, "shared memory budget");
    return launch_pdl(pts::w8a16_pair_ts_kernel, dim3(2 * clusters, 1, 1), dim3(pts::kThreads), pts::Smem::kTotal, st,
                      p);
}

}  // namespace npub

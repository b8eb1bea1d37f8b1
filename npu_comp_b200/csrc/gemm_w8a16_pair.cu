// Persistent W8A16 GEMM on 2-CTA tensor-core pairs (tcgen05 cta_group::2).
//
//   C[t, n] = fp16( alpha * scale[n] * sum_k A[t, k] * Wq[n, k] )  (+ R[t, n])
//
// A cluster of two CTAs on two SMs computes a 256 x BT tile of D = Wq * A^T:
// CTA r of the pair owns weight rows [a0 + 128 r, a0 + 128 r + 128) (the MMA's
// M side; its TMEM holds those D rows) and loads half of the token tile,
// rows [b0 + r BT/2, b0 + (r+1) BT/2) (the MMA's N side).  Every SM thus
// streams 128 int8 weight rows and BT/2 fp16 token rows per K step -- 24 KB at
// BT = 256 for 2*256*256*64 FLOP per pair -- which is what lets a deep TMA ring
// cover L2 latency.
//
// Roles per CTA (256 + 128 x converter groups threads):
//   warp 0      TMA producer: int8 weight tile -> own barrier full_a[s];
//               token half-tile -> the even CTA's barrier full_b[s]
//   warp 1      TMEM allocator (both CTAs); MMA issuer (even CTA only)
//   warps 4-7   epilogue: TMEM -> registers -> scale/residual -> global
//   warps 8+    converters in groups of four warps that take K steps in turn:
//               int8 stage -> fp16 128-byte-swizzled stage, then an arrive on
//               the even CTA's conv[c]
// The accumulator is double-buffered in TMEM (2 x BT columns), so the epilogue
// of one tile runs under the main loop of the next.  Cross-CTA signalling uses
// mapa + remote arrive and one commit per destination barrier; no TMA
// multicast is used anywhere.
//
// Reference semantics: the NPU matmul (_poc/mysim.cpp:109-113,
// b_program_examples/npu.py:41-47) with float32 accumulation and an fp16 store;
// the int8 weights and per-output-channel fp16 scales are the W8A16 scheme.
#include "common.cuh"
#include "gemm_tc.h"
#include "gemm_w8a16_pair.h"

#include <mutex>

namespace npub {

namespace pair {

template <int G>
constexpr int threads_for() { return 256 + 128 * G; }
constexpr int BK = kPairBK;       // K per stage
constexpr int KCH = kPairKch;     // 64-wide swizzled chunks per stage
constexpr int UMMA_K = 16;
constexpr int kRowsPerCta = 128;  // weight rows per CTA (MMA M = 256 per pair)

template <int BT, int STAGES, int CSTAGES>
struct Smem {
    static constexpr int kBhChunk = (BT / 2) * 64 * 2;  // one 64-wide chunk of the token half-tile
    static constexpr int kBh = KCH * kBhChunk;          // fp16 token half-tile per stage
    static constexpr int kA16Chunk = kRowsPerCta * 64 * 2;
    static constexpr int kA16 = KCH * kA16Chunk;
    static constexpr int kA8 = kRowsPerCta * BK;
    static constexpr int kBars = 8 * (3 * STAGES + 2 * CSTAGES + 4) + 16;
    static constexpr int kTotal = STAGES * (kBh + kA8) + CSTAGES * kA16 + kBars + 1024;
};

// 16 int8 -> 16 fp16, exact: (q ^ 0x80) placed in the mantissa of 1024.0, minus 1152.
__device__ __forceinline__ void cvt16(uint4 raw, uint4& lo, uint4& hi) {
    const uint32_t w0 = raw.x ^ 0x80808080u, w1 = raw.y ^ 0x80808080u, w2 = raw.z ^ 0x80808080u,
                   w3 = raw.w ^ 0x80808080u;
    lo = make_uint4(f16x2_sub1152(i8_perm_lo(w0)), f16x2_sub1152(i8_perm_hi(w0)), f16x2_sub1152(i8_perm_lo(w1)), f16x2_sub1152(i8_perm_hi(w1)));
    hi = make_uint4(f16x2_sub1152(i8_perm_lo(w2)), f16x2_sub1152(i8_perm_hi(w2)), f16x2_sub1152(i8_perm_lo(w3)), f16x2_sub1152(i8_perm_hi(w3)));
}

__device__ __forceinline__ void set_err(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

struct TileCoord {
    int a0, b0, split, kt0, nk;
};

// Without split-K the tiles go in bands of p.band token tiles: within a band
// the weight pairs in turn, each against every token tile of the band.  The
// ~74 tiles in flight then share a few weight pairs and one band of tokens
// (at most ~24 MB, sized on the host from K), so at 32768 tokens the weights
// come from HBM once per band instead of once per token tile.
__device__ __forceinline__ TileCoord tile_coord(const PairParams& p, int tile, int BT) {
    TileCoord c;
    int ap, bi;
    if (p.splits == 1) {
        const int per_band = p.band * p.n_apairs;
        const int band = tile / per_band;
        const int r = tile - band * per_band;
        const int nb = min(p.band, p.n_btiles - band * p.band);  // token tiles in this band
        ap = r / nb;
        bi = band * p.band + r % nb;
        c.split = 0;
    } else {
        ap = tile % p.n_apairs;
        const int rest = tile / p.n_apairs;
        bi = rest % p.n_btiles;
        c.split = rest / p.n_btiles;
    }
    c.a0 = ap * 2 * kRowsPerCta;
    c.b0 = bi * BT;
    c.kt0 = c.split * p.k_tiles_per_split;
    const int kt1 = min(p.k_tiles, c.kt0 + p.k_tiles_per_split);
    c.nk = kt1 > c.kt0 ? kt1 - c.kt0 : 0;
    return c;
}

template <int BT, int STAGES, int CSTAGES, int G>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(threads_for<G>(), 1)
    w8a16_pair_kernel(const __grid_constant__ PairParams p) {
    pdl_trigger();
    using L = Smem<BT, STAGES, CSTAGES>;
    static_assert(STAGES % G == 0 && CSTAGES >= G && CSTAGES >= 2, "see kPairStages*: converter groups take turns");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sB = smem;                            // STAGES x kBh   (1024-aligned)
    uint8_t* sA16 = sB + STAGES * L::kBh;          // CSTAGES x kA16
    uint8_t* sA8 = sA16 + CSTAGES * L::kA16;       // STAGES x kA8
    uint64_t* bars = reinterpret_cast<uint64_t*>(sA8 + STAGES * L::kA8);
    uint64_t* full_a = bars;                       // [STAGES] local int8 tile landed
    uint64_t* full_b = full_a + STAGES;            // [STAGES] (even CTA) both token halves landed
    uint64_t* empty = full_b + STAGES;             // [STAGES] pair MMA done with the stage
    uint64_t* conv = empty + STAGES;               // [CSTAGES] (even CTA) both CTAs converted
    uint64_t* c_empty = conv + CSTAGES;            // [CSTAGES] pair MMA done with the fp16 stage
    uint64_t* acc_full = c_empty + CSTAGES;        // [2] accumulator buffer ready
    uint64_t* acc_empty = acc_full + 2;            // [2] (even CTA) both epilogues drained the buffer
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int cid = (int)cluster_id_x(), ncl = (int)nclusters_x();

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_a[s], 1);
            mbar_init(&full_b[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int c = 0; c < CSTAGES; ++c) {
            mbar_init(&conv[c], 8);  // 2 CTAs x 4 converter warps
            mbar_init(&c_empty[c], 1);
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
        tmem_alloc_pair(tmem_slot, 2 * BT);
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
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            uint32_t g = 0;
            int issued = 0;
            const uint32_t full_b0 = mapa_shared(smem_u32(&full_b[0]), 0);
            for (int tile = cid; tile < p.n_tiles && !*abort_flag; tile += ncl) {
                const TileCoord tc = tile_coord(p, tile, BT);
                const int arow = tc.a0 + (int)rank * kRowsPerCta;
                const int brow = tc.b0 + (int)rank * (BT / 2);
                for (int i = 0; i < tc.nk; ++i, ++g) {
                    const int s = (int)(g % STAGES);
                    const uint32_t ph = (g / STAGES) & 1u;
                    if (!mbar_wait_cluster_bounded(&empty[s], ph ^ 1u, abort_flag)) {
                        *abort_flag = 1;
                        set_err(p.err, 0x201);
                        break;
                    }
                    const int k = (tc.kt0 + i) * BK;
                    mbar_arrive_expect_tx(&full_a[s], (uint32_t)L::kA8);
                    if (leader) mbar_arrive_expect_tx(&full_b[s], (uint32_t)(2 * L::kBh));
                    tma_load_3d(sA8 + s * L::kA8, &p.tmW, &full_a[s], k, arow, 0);
#pragma unroll
                    for (int ch = 0; ch < KCH; ++ch)
                        tma_load_3d_pair(sB + s * L::kBh + ch * L::kBhChunk, &p.tmX, full_b0 + (uint32_t)s * 8u,
                                         k + 64 * ch, brow, 0);
                    ++issued;
                }
            }
            // Drain: the last int8 loads of every stage have landed before exit
            // (token loads are awaited by the MMA issuer or time out there).
            for (uint32_t j = 0; j < (uint32_t)STAGES && (int)j < issued; ++j) {
                const uint32_t gg = g - 1 - j;
                const int s = (int)(gg % STAGES);
                if (!mbar_wait_cluster_bounded(&full_a[s], (gg / STAGES) & 1u, no_abort, 200000000ull))
                    set_err(p.err, 0x202);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (leader && lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(2 * kRowsPerCta, BT);
            const uint32_t peer = 1u;
            uint32_t g = 0, t = 0;
            bool ok = true;
            for (int tile = cid; tile < p.n_tiles && ok; tile += ncl, ++t) {
                const TileCoord tc = tile_coord(p, tile, BT);
                const uint32_t b = t & 1u, bph = (t >> 1) & 1u;
                if (!mbar_wait_cluster_bounded(&acc_empty[b], bph ^ 1u, abort_flag)) {
                    ok = false;
                    set_err(p.err, 0x203);
                    break;
                }
                tc_fence_after();
                const uint32_t dcol = tmem + b * (uint32_t)BT;
                for (int i = 0; i < tc.nk; ++i, ++g) {
                    const int s = (int)(g % STAGES);
                    const uint32_t ph = (g / STAGES) & 1u;
                    const int c = (int)(g % CSTAGES);
                    const uint32_t cph = (g / CSTAGES) & 1u;
                    if (!mbar_wait_cluster_bounded(&full_b[s], ph, abort_flag) ||
                        !mbar_wait_cluster_bounded(&conv[c], cph, abort_flag)) {
                        ok = false;
                        set_err(p.err, 0x204);
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int ch = 0; ch < KCH; ++ch) {
                        const uint32_t abase = smem_u32(sA16 + c * L::kA16 + ch * L::kA16Chunk);
                        const uint32_t bbase = smem_u32(sB + s * L::kBh + ch * L::kBhChunk);
#pragma unroll
                        for (int kk = 0; kk < 64 / UMMA_K; ++kk)
                            tc_mma_f16_pair(dcol, umma_desc_sw128(abase + kk * UMMA_K * 2),
                                            umma_desc_sw128(bbase + kk * UMMA_K * 2), idesc,
                                            (i > 0 || ch > 0 || kk > 0) ? 1u : 0u);
                    }
                    tc_commit_pair(smem_u32(&empty[s]));
                    tc_commit_pair(mapa_shared(smem_u32(&empty[s]), peer));
                    tc_commit_pair(smem_u32(&c_empty[c]));
                    tc_commit_pair(mapa_shared(smem_u32(&c_empty[c]), peer));
                }
                if (!ok) break;
                tc_commit_pair(smem_u32(&acc_full[b]));
                tc_commit_pair(mapa_shared(smem_u32(&acc_full[b]), peer));
            }
            if (!ok) *abort_flag = 1;
        }
    } else if (warp >= 8) {
        // ------------------------------------------------------------ converters
        const int grp = (warp - 8) >> 2;             // converter group
        const int t = (threadIdx.x - 256) & 127;     // 0..127 within the group
        const uint32_t conv0 = mapa_shared(smem_u32(&conv[0]), 0);
        uint32_t g = 0;
        bool ok = true;
        for (int tile = cid; tile < p.n_tiles && ok; tile += ncl) {
            const TileCoord tc = tile_coord(p, tile, BT);
            for (int i = 0; i < tc.nk; ++i, ++g) {
                if ((int)(g % G) != grp) continue;
                const int s = (int)(g % STAGES);
                const uint32_t ph = (g / STAGES) & 1u;
                const int c = (int)(g % CSTAGES);
                const uint32_t cph = (g / CSTAGES) & 1u;
                if (!mbar_wait_cluster_bounded(&full_a[s], ph, abort_flag) ||
                    !mbar_wait_cluster_bounded(&c_empty[c], cph ^ 1u, abort_flag)) {
                    ok = false;
                    *abort_flag = 1;
                    set_err(p.err, 0x205);
                    break;
                }
                const uint8_t* a8 = sA8 + s * L::kA8;
                uint8_t* a16 = sA16 + c * L::kA16;
#pragma unroll
                for (int j = 0; j < 4 * KCH; ++j) {  // 16 int8 per task, 4*KCH tasks per row
                    const int task = t + 128 * j;
                    const int row = task / (4 * KCH), q = task % (4 * KCH);
                    const uint4 raw = *reinterpret_cast<const uint4*>(a8 + row * BK + q * 16);
                    uint4 lo, hi;
                    cvt16(raw, lo, hi);
                    const int sw = row & 7, qq = q & 3;
                    uint8_t* dst = a16 + (q >> 2) * L::kA16Chunk + row * 128;
                    *reinterpret_cast<uint4*>(dst + (((2 * qq) ^ sw) << 4)) = lo;
                    *reinterpret_cast<uint4*>(dst + (((2 * qq + 1) ^ sw) << 4)) = hi;
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(conv0 + (uint32_t)c * 8u);
            }
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------ epilogue
        const int wq = warp & 3;
        const uint32_t accE0 = mapa_shared(smem_u32(&acc_empty[0]), 0);
        uint32_t t = 0;
        for (int tile = cid; tile < p.n_tiles; tile += ncl, ++t) {
            const TileCoord tc = tile_coord(p, tile, BT);
            const uint32_t b = t & 1u, bph = (t >> 1) & 1u;
            bool have = mbar_wait_cluster_bounded(&acc_full[b], bph, abort_flag);
            if (!have) set_err(p.err, 0x206);
            tc_fence_after();
            have = __all_sync(0xffffffffu, have && tc.nk > 0);
            const int a = tc.a0 + (int)rank * kRowsPerCta + wq * 32 + lane;
            const bool arow = a < p.N;
            float sc = 1.0f;
            if (!p.out_f32) sc = p.alpha * ((p.scale && arow) ? __half2float(p.scale[a]) : 1.0f);
            const int64_t obase = p.out_f32 ? (int64_t)tc.split * p.M * p.N + a : (int64_t)a;
            for (int c0 = 0; c0 < BT; c0 += 16) {
                if (tc.b0 + c0 >= p.M) break;  // warp-uniform
                float v[16];
                if (have) {
                    tmem_ld16(tmem + ((uint32_t)(wq * 32) << 16) + b * (uint32_t)BT + (uint32_t)c0, v);
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = 0.0f;
                }
                const int tb = tc.b0 + c0;
                if (p.swiglu && !p.out_f32) {
                    // gate row 2c and up row 2c + 1 sit in adjacent lanes (see
                    // the stream-K kernel): the even lane stores channel c
                    float gu[16], o[8];
#pragma unroll
                    for (int j = 0; j < 16; ++j) gu[j] = __half2float(__float2half_rn(v[j] * sc));
                    int t0;
                    swiglu_pair16(gu, lane, o, &t0);
                    if (arow) {
                        __half* dst = p.C + a / 2;
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            if (tb + t0 + j < p.M) dst[(int64_t)(tb + t0 + j) * p.ldc] = __float2half_rn(o[j]);
                    }
                    continue;
                }
                if (!arow) continue;
                if (p.out_f32) {
                    float* o = p.part + obase;
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (tb + j < p.M) o[(int64_t)(tb + j) * p.N] = v[j];
                } else {
                    __half* o = p.C + obase;
                    // all residual loads are issued before the first store (the two may
                    // alias as far as the compiler knows, which would serialise them)
                    float rv[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        rv[j] = (p.R && tb + j < p.M) ? __half2float(__ldg(p.R + (int64_t)(tb + j) * p.ldr + a)) : 0.0f;
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (tb + j < p.M) o[(int64_t)(tb + j) * p.ldc] = __float2half_rn(v[j] * sc + rv[j]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(accE0 + b * 8u);
        }
    }

    // Lane 0 alone ran some warps' role loops: a thread-counting barrier.
    tc_fence_before();
    cta_sync_divergent();
    cluster_sync();  // no CTA leaves while its peer may still signal or read it
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 2 * BT);
    }
}

// ---------------------------------------------------------------- host side

template <int BT, int STAGES, int CSTAGES, int G>
static int launch(const PairParams& p, int max_clusters, cudaStream_t st) {
    using L = Smem<BT, STAGES, CSTAGES>;
    static_assert(L::kTotal <= 232448, "shared memory budget");
    auto kern = w8a16_pair_kernel<BT, STAGES, CSTAGES, G>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
    if (e != cudaSuccess) {
        npub_internal_set_cuda_error(e);
        return NPUB_ERR_CUDA;
    }
    int clusters = p.n_tiles < max_clusters ? p.n_tiles : max_clusters;
    if (clusters < 1) clusters = 1;
    return launch_pdl(kern, dim3(2 * clusters, 1, 1), dim3(threads_for<G>()), L::kTotal, st, p);
}

static std::mutex g_mu;
static int g_max_clusters[64][3];

template <int BT, int STAGES, int CSTAGES, int G>
static int max_clusters_for(int dev, int slot) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_max_clusters[dev][slot] > 0) return g_max_clusters[dev][slot];
    using L = Smem<BT, STAGES, CSTAGES>;
    auto kern = w8a16_pair_kernel<BT, STAGES, CSTAGES, G>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 256, 1, 1);
    cfg.blockDim = dim3(threads_for<G>(), 1, 1);
    cfg.dynamicSmemBytes = L::kTotal;
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
    g_max_clusters[dev][slot] = n;
    return n;
}

}  // namespace pair

int pair_bt(int M) { return M <= 64 ? 64 : (M <= 128 ? 128 : 256); }

// Splits of K that fill whole waves of pair clusters.
int pair_splits(int tiles, int k_tiles, int clusters) {
    if (tiles >= clusters || k_tiles < 8) return 1;
    int best = 1;
    double best_t = 1e30;
    for (int s = 1; s <= 16 && k_tiles / s >= 4; ++s) {
        const int waves = (tiles * s + clusters - 1) / clusters;
        const double t = waves * ((double)k_tiles / s + 3.0) + (s > 1 ? 1.0 + 0.25 * s : 0.0);
        if (t < best_t - 1e-9) {
            best_t = t;
            best = s;
        }
    }
    return best;
}

static int cur_device() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= 64) d = 0;
    return d;
}

static int clusters_for_bt(int bt) {
    const int dev = cur_device();
    switch (bt) {
        case 64: return pair::max_clusters_for<64, kPairStages64, kPairCStages64, kPairGroups64>(dev, 0);
        case 128: return pair::max_clusters_for<128, kPairStages128, kPairCStages, kPairConvGroups>(dev, 1);
        default: return pair::max_clusters_for<256, kPairStages256, kPairCStages, kPairConvGroups>(dev, 2);
    }
}

size_t w8a16_pair_workspace(int M, int N, int K) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    const int bt = pair_bt(M);
    const int tiles = ((N + 255) / 256) * ((M + bt - 1) / bt);
    const int k_tiles = (K + kPairBK - 1) / kPairBK;
    const int s = pair_splits(tiles, k_tiles, clusters_for_bt(bt));
    return s > 1 ? (size_t)s * M * N * sizeof(float) : 0;
}

// Fills the scheduling fields of p and launches.  When split > 1 the kernel
// writes fp32 partials to ws and the caller reduces them.
int w8a16_pair_run(PairParams& p, int M, int N, int K, cudaStream_t st) {
    const int bt = pair_bt(M);
    p.M = M;
    p.N = N;
    p.k_tiles = (K + kPairBK - 1) / kPairBK;
    p.n_apairs = (N + 255) / 256;
    p.n_btiles = (M + bt - 1) / bt;
    const int clusters = clusters_for_bt(bt);
    const int splits = p.out_f32 ? pair_splits(p.n_apairs * p.n_btiles, p.k_tiles, clusters) : 1;
    p.k_tiles_per_split = (p.k_tiles + splits - 1) / splits;
    p.splits = (p.k_tiles + p.k_tiles_per_split - 1) / p.k_tiles_per_split;
    p.n_tiles = p.n_apairs * p.n_btiles * p.splits;
    // token tiles per band: ~24 MB of tokens (8 tiles of 256 at K = 4096, 4 at K = 11008)
    const int64_t tile_bytes = (int64_t)bt * K * 2;
    const int64_t band = (int64_t)(24 << 20) / (tile_bytes > 0 ? tile_bytes : 1);
    p.band = (int)(band < 1 ? 1 : (band > 8 ? 8 : band));
    p.err = npub_internal_device_error_word();
    switch (bt) {
        case 64: return pair::launch<64, kPairStages64, kPairCStages64, kPairGroups64>(p, clusters, st);
        case 128: return pair::launch<128, kPairStages128, kPairCStages, kPairConvGroups>(p, clusters, st);
        default: return pair::launch<256, kPairStages256, kPairCStages, kPairConvGroups>(p, clusters, st);
    }
}

int w8a16_pair_splits(int M, int N, int K) {
    const int bt = pair_bt(M);
    const int tiles = ((N + 255) / 256) * ((M + bt - 1) / bt);
    return pair_splits(tiles, (K + kPairBK - 1) / kPairBK, clusters_for_bt(bt));
}

}  // namespace npub

// Fused causal flash attention (prefill) for head_dim 128 on sm_100a.
//
// Per CTA: 128 query rows of one (sequence, head).  For each block of 128
// keys j (up to the causal diagonal):
//   S_j = Q K_j^T                 tcgen05.mma, fp32 accumulator in TMEM
//   P_j = exp2(S_j*scale*log2e - m_j)   one softmax thread per query row (the
//                                 row lives in one TMEM lane), fp16 into a
//                                 128-byte-swizzled shared tile
//   O_j = P_j V_j                 tcgen05.mma, V read MN-major straight from
//                                 its [keys, head_dim] layout
//   o = o * exp2(m_{j-1} - m_j) + O_j      in the softmax thread's registers
// S and O are double-buffered in TMEM (4 x 128 columns) and K/V in a two-stage
// TMA ring, so the tensor core computes S_{j+1} and O_j while the softmax
// threads work on block j.  Grouped-query heads read K/V head h / group.
//
// Semantics: softmax(Q K^T * scale + causal mask) V per head, the attention of
// b_program_examples/llama_layer.py:114-137 and
// d_compiler/npu_compiler/legalize.py:117-127, in the max-subtracted form of
// d_compiler/npu_compiler/model.py:145-150 (masked keys contribute exactly 0,
// as exp(-30000) does in the reference).
//
// Roles (320 threads): warp 0 TMA producer, warp 1 TMEM allocator + MMA
// issuer, warps 2-9 softmax / output.  Warp w reads TMEM lanes 32*(w%4)..+31;
// warps w and w+4 share those rows and split the 128 columns, exchanging the
// row maximum through shared memory (pair mbarriers, bounded waits).
#include "common.cuh"
#include "gemm_tc.h"

namespace npub {
namespace fmha {

constexpr int HD = 128;
constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int kThreads = 320;
constexpr int kChunk = 128 * 64 * 2;      // 128 rows x 64 fp16 (one swizzled 128-byte row each)
constexpr int kTile = 2 * kChunk;         // 128 x 128 fp16
constexpr int kOffQ = 0;
constexpr int kOffK0 = kTile;             // stage s: K at kOffK0 + s*2*kTile, V right after it
constexpr int kOffP0 = 5 * kTile;         // P[0], P[1]
constexpr int kOffBar = 7 * kTile;
constexpr int kOffXch = kOffBar + 256;    // float [2 parities][2 halves][128 rows]
constexpr int kSmem = kOffXch + 2 * 2 * 128 * 4;  // dynamic shared memory is 1024-byte aligned (checked)

struct Params {
    CUtensorMap tmQ, tmK, tmV;  // (head_dim, heads, rows), box (64, 1, 128), 128-byte swizzle
    int T, heads, kv_heads, group, n_qtiles, causal;
    float scale_log2;
    __half* out;
    int64_t ldo;
    int* err;
};

__device__ __forceinline__ void set_err(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

__global__ void __launch_bounds__(kThreads, 1) fmha_fwd_kernel(const __grid_constant__ Params p) {
    pdl_trigger();
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    if (smem_u32(smem_raw) & 1023u) {  // the swizzled tiles need 1024-byte alignment
        if (threadIdx.x == 0) set_err(p.err, 0x300);
        return;
    }
    uint8_t* smem = smem_raw;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint64_t* q_full = bars;            // 1
    uint64_t* k_full = bars + 1;        // [2]
    uint64_t* v_full = bars + 3;        // [2]
    uint64_t* kv_empty = bars + 5;      // [2]
    uint64_t* s_full = bars + 7;        // [2]
    uint64_t* s_free = bars + 9;        // [2]
    uint64_t* p_full = bars + 11;       // [2]
    uint64_t* p_free = bars + 13;       // [2]
    uint64_t* o_full = bars + 15;       // [2]
    uint64_t* o_free = bars + 17;       // [2]
    uint64_t* mma_done = bars + 19;     // 1
    uint64_t* pair_bar = bars + 20;     // [4] the two softmax warps of a lane quarter
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 24);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qt = p.n_qtiles - 1 - (int)blockIdx.x;  // longest causal rows first
    const int h = blockIdx.y, b = blockIdx.z;
    const int kvh = h / p.group;
    const int q0 = qt * BQ;
    const int row0 = b * p.T;
    const int kv_end = p.causal ? min(p.T, q0 + BQ) : p.T;
    const int nblk = (kv_end + BKV - 1) / BKV;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&kv_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 8);
            mbar_init(&p_full[i], 8);
            mbar_init(&p_free[i], 1);
            mbar_init(&o_full[i], 1);
            mbar_init(&o_free[i], 8);
        }
        mbar_init(mma_done, 1);
        for (int i = 0; i < 4; ++i) mbar_init(&pair_bar[i], 2);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&p.tmQ);
        prefetch_tmap(&p.tmK);
        prefetch_tmap(&p.tmV);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    cta_sync_divergent();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    int never = 0;
    volatile int* no_abort = &never;
    pdl_wait();

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, (uint32_t)kTile);
            tma_load_3d(smem + kOffQ, &p.tmQ, q_full, 0, h, row0 + q0);
            tma_load_3d(smem + kOffQ + kChunk, &p.tmQ, q_full, 64, h, row0 + q0);
            int issued = 0;
            for (int j = 0; j < nblk; ++j) {
                const int s = j & 1;
                const uint32_t ph = (uint32_t)(j >> 1) & 1u;
                if (!mbar_wait_bounded(&kv_empty[s], ph ^ 1u, abort_flag)) {
                    *abort_flag = 1;
                    set_err(p.err, 0x301);
                    break;
                }
                uint8_t* ks = smem + kOffK0 + s * 2 * kTile;
                uint8_t* vs = ks + kTile;
                const int r = row0 + j * BKV;
                mbar_arrive_expect_tx(&k_full[s], (uint32_t)kTile);
                tma_load_3d(ks, &p.tmK, &k_full[s], 0, kvh, r);
                tma_load_3d(ks + kChunk, &p.tmK, &k_full[s], 64, kvh, r);
                mbar_arrive_expect_tx(&v_full[s], (uint32_t)kTile);
                tma_load_3d(vs, &p.tmV, &v_full[s], 0, kvh, r);
                tma_load_3d(vs + kChunk, &p.tmV, &v_full[s], 64, kvh, r);
                ++issued;
            }
            if (!mbar_wait_bounded(q_full, 0, no_abort, 200000000ull)) set_err(p.err, 0x302);
            for (int j = issued - 1; j >= 0 && j >= issued - 2; --j) {
                const uint32_t ph = (uint32_t)(j >> 1) & 1u;
                if (!mbar_wait_bounded(&k_full[j & 1], ph, no_abort, 200000000ull) ||
                    !mbar_wait_bounded(&v_full[j & 1], ph, no_abort, 200000000ull))
                    set_err(p.err, 0x302);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc_s = umma_idesc_f16(BQ, BKV);
            constexpr uint32_t idesc_o = umma_idesc_f16_bmn(BQ, HD);
            bool ok = mbar_wait_bounded(q_full, 0, abort_flag);
            const uint32_t qa = smem_u32(smem + kOffQ);
            for (int j = 0; ok && j <= nblk; ++j) {
                if (j < nblk) {  // S_j = Q K_j^T into S[j&1]
                    const int s = j & 1;
                    const uint32_t ph = (uint32_t)(j >> 1) & 1u;
                    ok = mbar_wait_bounded(&k_full[s], ph, abort_flag) &&
                         mbar_wait_bounded(&s_free[s], ph ^ 1u, abort_flag);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t ka = smem_u32(smem + kOffK0 + s * 2 * kTile);
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk) {
                        const uint32_t off = (uint32_t)((kk >> 2) * kChunk + (kk & 3) * 32);
                        tc_mma_f16(tmem + (uint32_t)(s * 128), umma_desc_sw128(qa + off), umma_desc_sw128(ka + off),
                                   idesc_s, kk > 0 ? 1u : 0u);
                    }
                    tc_commit(&s_full[s]);
                }
                if (j >= 1) {  // O_{j-1} = P_{j-1} V_{j-1} into O[(j-1)&1]
                    const int jj = j - 1, s = jj & 1;
                    const uint32_t ph = (uint32_t)(jj >> 1) & 1u;
                    ok = mbar_wait_bounded(&p_full[s], ph, abort_flag) &&
                         mbar_wait_bounded(&v_full[s], ph, abort_flag) &&
                         mbar_wait_bounded(&o_free[s], ph ^ 1u, abort_flag);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t pa = smem_u32(smem + kOffP0 + s * kTile);
                    const uint32_t va = smem_u32(smem + kOffK0 + s * 2 * kTile + kTile);
#pragma unroll
                    for (int kk = 0; kk < BKV / 16; ++kk) {
                        const uint32_t aoff = (uint32_t)((kk >> 2) * kChunk + (kk & 3) * 32);
                        tc_mma_f16(tmem + 256u + (uint32_t)(s * 128), umma_desc_sw128(pa + aoff),
                                   umma_desc_sw128_mn(va + (uint32_t)kk * 2048u, (uint32_t)kChunk, 1024u), idesc_o,
                                   kk > 0 ? 1u : 0u);
                    }
                    tc_commit(&o_full[s]);
                    tc_commit(&p_free[s]);
                    tc_commit(&kv_empty[s]);
                }
            }
            if (!ok) {
                *abort_flag = 1;
                set_err(p.err, 0x303);
            }
            tc_commit(mma_done);  // every MMA issued above completes before TMEM is freed
            if (!mbar_wait_bounded(mma_done, 0, no_abort, 200000000ull)) set_err(p.err, 0x304);
        }
    } else {
        // ---------------------------------------------------------------- softmax / output
        const int wq = warp & 3;
        const int hf = (warp - 2) >> 2;        // column half handled by this warp
        const int col0 = hf * 64;
        const int r = wq * 32 + lane;          // row of the query tile == TMEM lane
        const int q_abs = q0 + r;
        const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
        float* xch = reinterpret_cast<float*>(smem + kOffXch);
        uint64_t* pb = &pair_bar[wq];
        float o[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) o[i] = 0.0f;
        float m = -INFINITY, l = 0.0f, corr_prev = 1.0f;
        bool ok = true;
        int rounds = 0;  // completed pair exchanges (phase of pb)
        for (int j = 0; j <= nblk && ok; ++j) {
            float corr = 1.0f;
            if (j < nblk) {
                const int s = j & 1;
                const uint32_t ph = (uint32_t)(j >> 1) & 1u;
                ok = __all_sync(0xffffffffu, mbar_wait_bounded(&s_full[s], ph, abort_flag));
                if (!ok) break;
                tc_fence_after();
                uint32_t sv[64];
                tmem_ld64(tmem + lane_off + (uint32_t)(s * 128 + col0), sv);
                // the S buffer can be overwritten by S_{j+2} once every warp has read it
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_free[s]);
                float x[64];
                const int kbase = j * BKV + col0;
                const bool need_mask = (p.causal && j * BKV + BKV - 1 > q0) || j * BKV + BKV > p.T;  // CTA-uniform
                if (need_mask) {
#pragma unroll
                    for (int e = 0; e < 64; ++e) {
                        const int key = kbase + e;
                        const bool msk = (p.causal && key > q_abs) || key >= p.T;
                        x[e] = msk ? -INFINITY : __uint_as_float(sv[e]) * p.scale_log2;
                    }
                } else {
#pragma unroll
                    for (int e = 0; e < 64; ++e) x[e] = __uint_as_float(sv[e]) * p.scale_log2;
                }
                float m4[4] = {x[0], x[1], x[2], x[3]};
#pragma unroll
                for (int e = 4; e < 64; ++e) m4[e & 3] = fmaxf(m4[e & 3], x[e]);
                const float lmax = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
                // exchange the half-row maxima with the partner warp
                float* xs = xch + (j & 1) * 256;
                xs[hf * 128 + r] = lmax;
                __syncwarp();
                if (lane == 0) mbar_arrive(pb);
                ok = __all_sync(0xffffffffu, mbar_wait_bounded(pb, (uint32_t)(rounds & 1), abort_flag));
                ++rounds;
                if (!ok) break;
                const float mx = fmaxf(m, fmaxf(lmax, xs[(1 - hf) * 128 + r]));
                corr = (mx == -INFINITY) ? 1.0f : ex2_approx(m - mx);
                ok = __all_sync(0xffffffffu, mbar_wait_bounded(&p_free[s], ph ^ 1u, abort_flag));
                if (!ok) break;
                uint8_t* prow = smem + kOffP0 + s * kTile + hf * kChunk + r * 128;
                const int sw = r & 7;
                float rs[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int pc = 0; pc < 8; ++pc) {  // 8 keys per 16-byte piece
                    uint32_t pk[4];
#pragma unroll
                    for (int e = 0; e < 8; e += 2) {
                        const float p0 = ex2_approx(x[pc * 8 + e] - mx);
                        const float p1 = ex2_approx(x[pc * 8 + e + 1] - mx);
                        rs[e >> 1] += p0 + p1;
                        __half2 hh = __floats2half2_rn(p0, p1);
                        pk[e >> 1] = *reinterpret_cast<uint32_t*>(&hh);
                    }
                    *reinterpret_cast<uint4*>(prow + ((pc ^ sw) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[s]);
                l = l * corr + ((rs[0] + rs[1]) + (rs[2] + rs[3]));
                m = mx;
            }
            if (j >= 1) {  // o = o * corr_{j-1} + O_{j-1}  (this warp's 64 output columns)
                const int jj = j - 1, s = jj & 1;
                const uint32_t ph = (uint32_t)(jj >> 1) & 1u;
                ok = __all_sync(0xffffffffu, mbar_wait_bounded(&o_full[s], ph, abort_flag));
                if (!ok) break;
                tc_fence_after();
                uint32_t ov[64];
                tmem_ld64(tmem + lane_off + 256u + (uint32_t)(s * 128 + col0), ov);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&o_free[s]);
#pragma unroll
                for (int e = 0; e < 64; ++e) o[e] = o[e] * corr_prev + __uint_as_float(ov[e]);
            }
            corr_prev = corr;
        }
        if (ok) {  // the row sum is split across the pair too
            float* xs = xch + (rounds & 1) * 256;
            xs[hf * 128 + r] = l;
            __syncwarp();
            if (lane == 0) mbar_arrive(pb);
            ok = __all_sync(0xffffffffu, mbar_wait_bounded(pb, (uint32_t)(rounds & 1), abort_flag));
            if (ok) l += xs[(1 - hf) * 128 + r];
        }
        if (!ok) {
            *abort_flag = 1;
            set_err(p.err, 0x305);
        } else if (q_abs < p.T) {
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            __half* dst = p.out + (int64_t)(row0 + q_abs) * p.ldo + (int64_t)h * HD + col0;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                uint32_t pk[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    __half2 hh = __floats2half2_rn(o[c * 8 + 2 * e] * inv, o[c * 8 + 2 * e + 1] * inv);
                    pk[e] = *reinterpret_cast<uint32_t*>(&hh);
                }
                *reinterpret_cast<uint4*>(dst + c * 8) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
        }
    }

    // Lane 0 alone ran some warps' role loops: a thread-counting barrier.
    tc_fence_before();
    cta_sync_divergent();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace fmha

// Fused path of npub_attention_prefill for head_dim 128 (no workspace).
int fmha_prefill(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv, void* out,
                 int64_t ldo, int batch, int tokens, int heads, int kv_heads, float scale, int causal,
                 cudaStream_t st) {
    using namespace fmha;
    Params p;
    memset(&p, 0, sizeof(p));
    const uint64_t rows = (uint64_t)batch * tokens;
    int rc = make_tmap_3d(&p.tmQ, false, q, HD, (uint64_t)heads, rows, HD, (uint64_t)ldq, 1, 128, true);
    if (rc) return rc;
    rc = make_tmap_3d(&p.tmK, false, k, HD, (uint64_t)kv_heads, rows, HD, (uint64_t)ldk, 1, 128, true);
    if (rc) return rc;
    rc = make_tmap_3d(&p.tmV, false, v, HD, (uint64_t)kv_heads, rows, HD, (uint64_t)ldv, 1, 128, true);
    if (rc) return rc;
    p.T = tokens;
    p.heads = heads;
    p.kv_heads = kv_heads;
    p.group = heads / kv_heads;
    p.n_qtiles = (tokens + BQ - 1) / BQ;
    p.causal = causal ? 1 : 0;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.out = reinterpret_cast<__half*>(out);
    p.ldo = ldo;
    p.err = npub_internal_device_error_word();
    cudaError_t e = cudaFuncSetAttribute(fmha_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) {
        npub_internal_set_cuda_error(e);
        return NPUB_ERR_CUDA;
    }
    return launch_pdl(fmha_fwd_kernel, dim3(p.n_qtiles, heads, batch), dim3(kThreads), kSmem, st, p);
}

}  // namespace npub

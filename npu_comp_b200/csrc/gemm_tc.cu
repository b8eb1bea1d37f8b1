// Tensor-core GEMM for sm_100a: TMA -> shared memory -> tcgen05.mma with the
// fp32 accumulator in tensor memory (TMEM) -> fused epilogue.
//
//   D[a, b] = sum_k Aop[a, k] * Bop[b, k]        (both operands K-major)
//
// One CTA computes a 128 x BT tile of D.  For the W8A16 matmul the A operand
// is the int8 weight matrix Wq [N, K]: TMA streams raw int8 tiles into shared
// memory, four converter warps turn them into fp16 in the 128-byte swizzled
// K-major layout the MMA reads, and the per-output-channel scale is applied in
// the epilogue, where row `a` of the tile is the output channel.  The B
// operand is the fp16 activation tile (BT token rows).  The same kernel with
// an fp16 A operand serves the fp16 matmul and the batched attention GEMMs
// (Q K^T and P V), where blockIdx.z is the head.
//
// Reference semantics: the NPU matmul C = A @ B with float32 accumulation and
// an fp16 store (_poc/mysim.cpp:109-113, b_program_examples/npu.py:41-47).
//
// Warp roles (256 threads):
//   warp 0      TMA producer (one elected lane)
//   warp 1      TMEM allocator + MMA issuer (one elected lane)
//   warps 4..7  int8 -> fp16 converters during the main loop, then the
//               epilogue (warp 4+i reads TMEM lanes 32i..32i+31)
#include "common.cuh"
#include "gemm_tc.h"
#include "gemm_w8a16_pair.h"
#include "gemm_w8a16_skinny.h"

#include <cudaTypedefs.h>

#include <mutex>

namespace npub {

constexpr int BM = 128;  // A rows per tile == TMEM lanes
constexpr int BK = 64;   // K per pipeline stage: one 128-byte row of fp16
constexpr int UMMA_K = 16;
constexpr int kThreads = 256;

template <bool A_I8, int BT, int STAGES>
struct GemmSmem {
    static constexpr int kB = BT * BK * 2;         // fp16 B stage
    static constexpr int kA16 = BM * BK * 2;       // fp16 A stage (MMA operand)
    static constexpr int kA8 = A_I8 ? BM * BK : 0; // raw int8 A stage
    static constexpr int kStage = kB + kA16 + kA8;
    static constexpr int kBarriers = 8 * (3 * STAGES + 1) + 16;
    static constexpr int kTotal = STAGES * kStage + kBarriers + 1024;  // + alignment slack
};

__device__ __forceinline__ uint32_t i8x4_to_f16x2_lo(uint32_t u) {
    // bytes b0,b1 of u (already xor 0x80) -> half2 {1024 + b0, 1024 + b1}
    return __byte_perm(u, 0x64646464u, 0x5140);
}
__device__ __forceinline__ uint32_t i8x4_to_f16x2_hi(uint32_t u) { return __byte_perm(u, 0x64646464u, 0x5342); }

__device__ __forceinline__ uint32_t hsub_1152(uint32_t h) {
    __half2 v = *reinterpret_cast<__half2*>(&h);
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152.0
    __half2 r = __hsub2(v, bias);
    return *reinterpret_cast<uint32_t*>(&r);
}

// 16 int8 values -> 16 fp16 values (exact: |q| <= 128 < 2048).
__device__ __forceinline__ void cvt16_i8_f16(uint4 raw, uint4& lo, uint4& hi) {
    uint32_t w[4] = {raw.x ^ 0x80808080u, raw.y ^ 0x80808080u, raw.z ^ 0x80808080u, raw.w ^ 0x80808080u};
    lo.x = hsub_1152(i8x4_to_f16x2_lo(w[0]));
    lo.y = hsub_1152(i8x4_to_f16x2_hi(w[0]));
    lo.z = hsub_1152(i8x4_to_f16x2_lo(w[1]));
    lo.w = hsub_1152(i8x4_to_f16x2_hi(w[1]));
    hi.x = hsub_1152(i8x4_to_f16x2_lo(w[2]));
    hi.y = hsub_1152(i8x4_to_f16x2_hi(w[2]));
    hi.z = hsub_1152(i8x4_to_f16x2_lo(w[3]));
    hi.w = hsub_1152(i8x4_to_f16x2_hi(w[3]));
}

__device__ __forceinline__ void set_error(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

template <bool A_I8, int BT, int STAGES>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ GemmParams p) {
    pdl_trigger();
    using L = GemmSmem<A_I8, BT, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sB = smem;                             // STAGES x kB   (1024-aligned: kB % 1024 == 0)
    uint8_t* sA16 = sB + STAGES * L::kB;            // STAGES x kA16
    uint8_t* sA8 = sA16 + STAGES * L::kA16;         // STAGES x kA8
    uint64_t* bars = reinterpret_cast<uint64_t*>(sA8 + STAGES * L::kA8);
    uint64_t* full = bars;                          // TMA landed
    uint64_t* conv = bars + STAGES;                 // int8 stage converted (A_I8)
    uint64_t* empty = bars + 2 * STAGES;            // MMA finished reading the stage
    uint64_t* accum = bars + 3 * STAGES;            // accumulator complete
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * STAGES + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int a0 = blockIdx.x * BM;
    const int b0 = blockIdx.y * BT;
    const int z = blockIdx.z / p.splits;
    const int split = blockIdx.z - z * p.splits;

    // Tiles wholly above the causal diagonal are never read: skip them.
    if (p.causal_mode == 1 && b0 > a0 + BM - 1 + p.causal_off) return;

    int kt0 = split * p.k_tiles_per_split;
    int kt1 = min(p.k_tiles, kt0 + p.k_tiles_per_split);
    if (p.causal_mode == 2) {
        int lim = a0 + BM + p.causal_off;
        lim = lim < 0 ? 0 : lim;
        kt1 = min(kt1, (lim + BK - 1) / BK);
    }
    const int nk = kt1 > kt0 ? kt1 - kt0 : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&conv[s], BM);  // one arrival per converter thread
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&p.tmA);
        prefetch_tmap(&p.tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, BT);
        tmem_relinquish();
    }
    tc_fence_before();
    cta_sync_divergent();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    int never = 0;
    volatile int* no_abort = &never;
    pdl_wait();

    const int zl = z % p.zmod, zh = z / p.zmod;
    const int a_bat = zl / p.za.div + zh * p.za.bat_hi;
    const int a_off = zh * p.za.zrow_hi + zl * p.za.zrow_lo;
    const int b_bat = zl / p.zb.div + zh * p.zb.bat_hi;
    const int b_off = zh * p.zb.zrow_hi + zl * p.zb.zrow_lo;
    if (warp == 0) {
        if (lane == 0 && nk > 0) {
            int issued = 0;
            for (int i = 0; i < nk; ++i) {
                const int s = i % STAGES;
                const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
                if (!mbar_wait_bounded(&empty[s], ph ^ 1u, abort_flag)) {
                    *abort_flag = 1;
                    set_error(p.err, 0x101);
                    break;
                }
                mbar_arrive_expect_tx(&full[s], (uint32_t)(L::kB + (A_I8 ? L::kA8 : L::kA16)));
                const int k = (kt0 + i) * BK;
                void* adst = A_I8 ? (void*)(sA8 + s * L::kA8) : (void*)(sA16 + s * L::kA16);
                if (p.a_row_dim == 1)
                    tma_load_3d(adst, &p.tmA, &full[s], k, a_off + a0, a_bat);
                else
                    tma_load_3d(adst, &p.tmA, &full[s], k, a_bat, a_off + a0);
                if (p.b_row_dim == 1)
                    tma_load_3d(sB + s * L::kB, &p.tmB, &full[s], k, b_off + b0, b_bat);
                else
                    tma_load_3d(sB + s * L::kB, &p.tmB, &full[s], k, b_bat, b_off + b0);
                ++issued;
            }
            // Drain: the last loads of every stage have landed before the CTA can exit.
            for (int i = issued - 1; i >= 0 && i >= issued - STAGES; --i) {
                const int s = i % STAGES;
                const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
                if (!mbar_wait_bounded(&full[s], ph, no_abort, 200000000ull)) set_error(p.err, 0x102);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && nk > 0) {
            constexpr uint32_t idesc = umma_idesc_f16(BM, BT);
            for (int i = 0; i < nk; ++i) {
                const int s = i % STAGES;
                const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
                if (!mbar_wait_bounded(A_I8 ? &conv[s] : &full[s], ph, abort_flag)) {
                    *abort_flag = 1;
                    set_error(p.err, 0x103);
                    break;
                }
                tc_fence_after();
                const uint32_t abase = smem_u32(sA16 + s * L::kA16);
                const uint32_t bbase = smem_u32(sB + s * L::kB);
#pragma unroll
                for (int kk = 0; kk < BK / UMMA_K; ++kk) {
                    const uint64_t ad = umma_desc_sw128(abase + kk * UMMA_K * 2);
                    const uint64_t bd = umma_desc_sw128(bbase + kk * UMMA_K * 2);
                    tc_mma_f16(tmem, ad, bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
                }
                tc_commit(&empty[s]);
            }
            tc_commit(accum);  // tracks every MMA issued above
        }
    } else if (warp >= 4) {
        const int t = threadIdx.x - 128;  // 0..127
        if (A_I8) {
            for (int i = 0; i < nk; ++i) {
                const int s = i % STAGES;
                const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
                if (!mbar_wait_bounded(&full[s], ph, abort_flag)) {
                    *abort_flag = 1;
                    set_error(p.err, 0x104);
                    break;
                }
                const uint8_t* a8 = sA8 + s * L::kA8;
                uint8_t* a16 = sA16 + s * L::kA16;
#pragma unroll
                for (int j = 0; j < (BM * BK / 16) / 128; ++j) {  // 4 chunks of 16 int8 per thread
                    const int task = t + 128 * j;
                    const int row = task >> 2, c = task & 3;
                    const uint4 raw = *reinterpret_cast<const uint4*>(a8 + row * BK + c * 16);
                    uint4 lo, hi;
                    cvt16_i8_f16(raw, lo, hi);
                    const int sw = row & 7;
                    *reinterpret_cast<uint4*>(a16 + row * 128 + (((2 * c) ^ sw) << 4)) = lo;
                    *reinterpret_cast<uint4*>(a16 + row * 128 + (((2 * c + 1) ^ sw) << 4)) = hi;
                }
                fence_proxy_async_smem();
                mbar_arrive(&conv[s]);
            }
        }
        // ---------------- epilogue: TMEM -> registers -> global
        bool have = nk > 0;
        if (have) {
            if (!mbar_wait_bounded(accum, 0, no_abort)) {
                set_error(p.err, 0x105);
                have = false;
            }
            tc_fence_after();
        }
        if (*abort_flag) have = false;
        have = __all_sync(0xffffffffu, have);  // tcgen05.ld below is warp-collective
        const int wq = warp & 3;
        const int a = a0 + wq * 32 + lane;
        const bool arow = a < p.a_rows;
        float sc = 1.0f;
        if (!p.out_f32) sc = p.alpha * ((p.a_scale && arow) ? __half2float(p.a_scale[a]) : 1.0f);
        const int64_t obase = (int64_t)a * p.o_sa + (int64_t)zl * p.o_zl + (int64_t)zh * p.o_zh +
                              (p.out_f32 ? (int64_t)split * p.o_split : 0);
        const int64_t rbase = (int64_t)a * p.r_sa + (int64_t)zl * p.r_zl + (int64_t)zh * p.r_zh;
        for (int c0 = 0; c0 < BT; c0 += 16) {
            if (b0 + c0 >= p.b_rows) break;  // warp-uniform
            float v[16];
            if (have) {
                tmem_ld16(tmem + ((uint32_t)(wq * 32) << 16) + (uint32_t)c0, v);
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = 0.0f;
            }
            if (!arow) continue;
            const int bb = b0 + c0;
            if (p.out_f32) {
                float* o = reinterpret_cast<float*>(p.out) + obase;
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (bb + j < p.b_rows) o[(int64_t)(bb + j) * p.o_sb] = v[j];
                continue;
            }
            __half* o = reinterpret_cast<__half*>(p.out) + obase;
            const bool vec = p.o_sb == 1 && bb + 16 <= p.b_rows && p.res == nullptr &&
                             ((reinterpret_cast<uintptr_t>(o + bb) & 15) == 0);
            if (vec) {
                uint32_t pk[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    __half2 h = __floats2half2_rn(v[2 * j] * sc, v[2 * j + 1] * sc);
                    pk[j] = *reinterpret_cast<uint32_t*>(&h);
                }
                uint4* dst = reinterpret_cast<uint4*>(o + bb);
                dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
            } else {
                float rv[16];  // residual loads first: stores may alias them as far as the compiler knows
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    rv[j] = (p.res && bb + j < p.b_rows) ? __half2float(__ldg(p.res + rbase + (int64_t)(bb + j) * p.r_sb))
                                                         : 0.0f;
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (bb + j < p.b_rows) o[(int64_t)(bb + j) * p.o_sb] = __float2half_rn(v[j] * sc + rv[j]);
            }
        }
    }

    // Lane 0 alone ran some warps' role loops: a thread-counting barrier.
    tc_fence_before();
    cta_sync_divergent();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, BT);
    }
}

// Split-K reduction: out[m, n] = fp16(alpha * scale[n] * sum_s part[s, m, n]) (+ res[m, n]).
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, int M, int N,
                                     const __half* __restrict__ scale, float alpha, const __half* __restrict__ res,
                                     int64_t ldr, __half* __restrict__ out, int64_t ldo) {
    pdl_trigger();
    pdl_wait();
    const int64_t total = (int64_t)M * N;
    const int64_t plane = total;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int m = (int)(i / N), n = (int)(i - (int64_t)m * N);
        float acc = 0.0f;
        for (int s = 0; s < splits; ++s) acc += part[s * plane + i];
        float x = acc * alpha * (scale ? __half2float(scale[n]) : 1.0f);
        if (res) x += __half2float(res[(int64_t)m * ldr + n]);
        out[(int64_t)m * ldo + n] = __float2half_rn(x);
    }
}

// Split-K reduction of a gate|up projection with interleaved rows (2c gate,
// 2c + 1 up) fused with SwiGLU: out [M, N/2].  g and u are rounded to fp16
// exactly as splitk_reduce_kernel would store them.
__global__ void splitk_reduce_swiglu_kernel(const float* __restrict__ part, int splits, int M, int N,
                                            const __half* __restrict__ scale, float alpha, __half* __restrict__ out,
                                            int64_t ldo) {
    pdl_trigger();
    pdl_wait();
    const int F = N / 2;
    const int64_t total = (int64_t)M * F;
    const int64_t plane = (int64_t)M * N;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int m = (int)(i / F), c = (int)(i - (int64_t)m * F);
        const int64_t e = (int64_t)m * N + 2 * c;
        float ga = 0.0f, ua = 0.0f;
        for (int s = 0; s < splits; ++s) {
            ga += part[s * plane + e];
            ua += part[s * plane + e + 1];
        }
        const float g = __half2float(__float2half_rn(ga * alpha * (scale ? __half2float(scale[2 * c]) : 1.0f)));
        const float u = __half2float(__float2half_rn(ua * alpha * (scale ? __half2float(scale[2 * c + 1]) : 1.0f)));
        out[(int64_t)m * ldo + c] = __float2half_rn(swiglu_f(g, u));
    }
}

// ------------------------------------------------------------------ host side

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;
static int g_num_sms[64];
static std::mutex g_sm_mu;

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return g_encode;
}

int num_sms() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lk(g_sm_mu);
    if (g_num_sms[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        g_num_sms[dev] = n;
    }
    return g_num_sms[dev];
}

int make_tmap_3d(CUtensorMap* m, bool int8, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                 uint64_t s2, uint32_t box1, uint32_t box2, bool swizzle128, uint32_t box0) {
    auto enc = encode_fn();
    if (!enc) return NPUB_ERR_CUDA;
    const int es = int8 ? 1 : 2;
    cuuint64_t gdim[3] = {d0, d1, d2};
    cuuint64_t gstride[2] = {s1 * es, s2 * es};
    cuuint32_t box[3] = {(cuuint32_t)box0, box1, box2};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, int8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                     const_cast<void*>(base), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? NPUB_OK : NPUB_ERR_INVALID_ARG;
}

template <bool A_I8, int BT, int STAGES>
static int launch_cfg(const GemmParams& p, int grid_x, int grid_y, int grid_z, cudaStream_t st) {
    using L = GemmSmem<A_I8, BT, STAGES>;
    static_assert(L::kTotal <= 232448, "shared memory budget");
    auto kern = gemm_tc_kernel<A_I8, BT, STAGES>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
    if (e != cudaSuccess) {
        npub_internal_set_cuda_error(e);
        return NPUB_ERR_CUDA;
    }
    return launch_pdl(kern, dim3(grid_x, grid_y, grid_z), dim3(kThreads), L::kTotal, st, p);
}

template <bool A_I8>
static int launch_bt(int bt, const GemmParams& p, int gx, int gy, int gz, cudaStream_t st) {
    switch (bt) {
        case 64: return launch_cfg<A_I8, 64, 6>(p, gx, gy, gz, st);
        case 128: return launch_cfg<A_I8, 128, 4>(p, gx, gy, gz, st);
        default: return launch_cfg<A_I8, 256, 3>(p, gx, gy, gz, st);
    }
}

int pick_bt(int b_rows) {
    if (b_rows <= 64) return 64;
    if (b_rows <= 128) return 128;
    return 256;
}

// Splits of the K loop that best fill whole waves of CTAs (1 CTA per SM).
int pick_splits(int tiles, int k_tiles) {
    const int sms = num_sms();
    if (tiles >= sms || k_tiles < 8) return 1;
    int best = 1;
    double best_t = 1e30;
    for (int s = 1; s <= 16 && k_tiles / s >= 4; ++s) {
        const int ctas = tiles * s;
        const int waves = (ctas + sms - 1) / sms;
        // time ~ waves * (k_tiles / s) k-steps + fixed cost per wave + reduce cost
        const double t = waves * ((double)k_tiles / s + 6.0) + (s > 1 ? 2.0 + 0.5 * s : 0.0);
        if (t < best_t - 1e-9) {
            best_t = t;
            best = s;
        }
    }
    return best;
}

int run_gemm(GemmParams& p, bool a_int8, int bt, int grid_x, int grid_y, int batch, cudaStream_t st) {
    p.err = npub_internal_device_error_word();
    const int gz = batch * p.splits;
    if (grid_x <= 0 || grid_y <= 0 || gz <= 0) return NPUB_OK;
    if (grid_y > 65535 || gz > 65535) return NPUB_ERR_UNSUPPORTED;
    return a_int8 ? launch_bt<true>(bt, p, grid_x, grid_y, gz, st) : launch_bt<false>(bt, p, grid_x, grid_y, gz, st);
}

// Shared host path of npub_w8a16_gemm / npub_f16_gemm:
// Aop = weights [N, K] (128-row side), Bop = activations [M, K] (token side).
static size_t linear_workspace(int M, int N, int K, bool w_int8) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    if (w_int8) {
        // every W8A16 workspace starts with the stream-K kernel's counter region
        if (w8a16_use_skinny(M, N, K)) return w8a16_skinny_workspace(M, N, K);
        const size_t pair = w8a16_pair_workspace(M, N, K);
        return pair ? kSkinnyCounterBytes + pair : 0;
    }
    const int bt = pick_bt(M);
    const int tiles = ((N + BM - 1) / BM) * ((M + bt - 1) / bt);
    const int k_tiles = (K + BK - 1) / BK;
    const int s = pick_splits(tiles, k_tiles);
    return s > 1 ? (size_t)s * M * N * sizeof(float) : 0;
}

// W8A16 on 2-CTA pairs: weights are the 256-row MMA side, tokens the BT side.
static int linear_w8a16_pair(const void* A, int64_t lda, const void* W, int64_t ldw, const void* scale, void* C,
                             int64_t ldc, const void* R, int64_t ldr, int M, int N, int K, float alpha, void* ws,
                             size_t ws_bytes, cudaStream_t st, int swiglu = 0) {
    PairParams p;
    memset(&p, 0, sizeof(p));
    const int bt = pair_bt(M);
    int rc = make_tmap_3d(&p.tmW, true, W, (uint64_t)K, (uint64_t)N, 1, (uint64_t)ldw, (uint64_t)ldw * N, 128, 1,
                          false, kPairBK);
    if (rc) return rc;
    rc = make_tmap_3d(&p.tmX, false, A, (uint64_t)K, (uint64_t)M, 1, (uint64_t)lda, (uint64_t)lda * M,
                      (uint32_t)(bt / 2), 1, true);
    if (rc) return rc;
    const int splits = w8a16_pair_splits(M, N, K);
    p.alpha = alpha;
    if (splits > 1) {
        // partials after the counter region, which only the stream-K kernel uses
        const size_t need = (size_t)splits * M * N * sizeof(float);
        if (!ws || ws_bytes < kSkinnyCounterBytes + need) return NPUB_ERR_WORKSPACE;
        ws = static_cast<uint8_t*>(ws) + kSkinnyCounterBytes;
        if (!npub_aligned(ws, 16)) return NPUB_ERR_INVALID_ARG;
        p.out_f32 = 1;
        p.part = reinterpret_cast<float*>(ws);
    } else {
        p.C = reinterpret_cast<__half*>(C);
        p.ldc = ldc;
        p.R = reinterpret_cast<const __half*>(R);
        p.ldr = ldr;
        p.scale = reinterpret_cast<const __half*>(scale);
        p.swiglu = swiglu;
    }
    rc = w8a16_pair_run(p, M, N, K, st);
    if (rc || p.splits == 1) return rc;
    const int64_t total = (int64_t)M * (swiglu ? N / 2 : N);
    int blocks = (int)((total + 255) / 256);
    const int cap = num_sms() * 8;
    if (blocks > cap) blocks = cap;
    if (swiglu)
        return launch_pdl(splitk_reduce_swiglu_kernel, dim3(blocks), dim3(256), 0, st,
                          reinterpret_cast<const float*>(ws), p.splits, M, N, reinterpret_cast<const __half*>(scale),
                          alpha, reinterpret_cast<__half*>(C), ldc);
    return launch_pdl(splitk_reduce_kernel, dim3(blocks), dim3(256), 0, st, reinterpret_cast<const float*>(ws), p.splits, M, N,
                                                 reinterpret_cast<const __half*>(scale), alpha,
                                                 reinterpret_cast<const __half*>(R), ldr, reinterpret_cast<__half*>(C),
                                                 ldc);
}

static int linear(bool w_int8, const void* A, int64_t lda, const void* W, int64_t ldw, const void* scale, void* C,
                  int64_t ldc, const void* R, int64_t ldr, int M, int N, int K, float alpha, void* ws, size_t ws_bytes,
                  void* stream) {
    NPUB_CHECK_ARG(M >= 0 && N >= 0 && K >= 0);
    if (M == 0 || N == 0) return NPUB_OK;
    NPUB_CHECK_ARG(A && W && C);
    NPUB_CHECK_ARG(K % 16 == 0 && K > 0);
    NPUB_CHECK_ARG(lda >= K && lda % 8 == 0 && npub_aligned(A, 16));
    NPUB_CHECK_ARG(ldw >= K && npub_aligned(W, 16));
    NPUB_CHECK_ARG(w_int8 ? (ldw % 16 == 0) : (ldw % 8 == 0));
    NPUB_CHECK_ARG(ldc >= N);
    NPUB_CHECK_ARG(!R || ldr >= N);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (w_int8 && w8a16_use_skinny(M, N, K))
        return w8a16_skinny_run(A, lda, W, ldw, scale, C, ldc, R, ldr, M, N, K, alpha, ws, ws_bytes, st);
    if (w_int8) return linear_w8a16_pair(A, lda, W, ldw, scale, C, ldc, R, ldr, M, N, K, alpha, ws, ws_bytes, st);

    GemmParams p;
    memset(&p, 0, sizeof(p));
    int rc = make_tmap_3d(&p.tmA, w_int8, W, (uint64_t)K, (uint64_t)N, 1, (uint64_t)ldw, (uint64_t)ldw * N, BM, 1,
                          !w_int8);
    if (rc) return rc;
    const int bt = pick_bt(M);
    rc = make_tmap_3d(&p.tmB, false, A, (uint64_t)K, (uint64_t)M, 1, (uint64_t)lda, (uint64_t)lda * M, bt, 1, true);
    if (rc) return rc;
    p.a_rows = N;
    p.b_rows = M;
    p.k_tiles = (K + BK - 1) / BK;
    p.a_row_dim = 1;
    p.b_row_dim = 1;
    zmap_plain(p);
    const int gx = (N + BM - 1) / BM, gy = (M + bt - 1) / bt;
    const int splits = pick_splits(gx * gy, p.k_tiles);
    p.k_tiles_per_split = (p.k_tiles + splits - 1) / splits;
    p.splits = (p.k_tiles + p.k_tiles_per_split - 1) / p.k_tiles_per_split;
    p.causal_mode = 0;
    p.alpha = alpha;
    if (p.splits > 1) {
        const size_t need = (size_t)p.splits * M * N * sizeof(float);
        if (!ws || ws_bytes < need) return NPUB_ERR_WORKSPACE;
        if (!npub_aligned(ws, 16)) return NPUB_ERR_INVALID_ARG;
        p.out = ws;
        p.out_f32 = 1;
        p.o_sa = 1;
        p.o_sb = N;
        p.o_split = (int64_t)M * N;
    } else {
        p.out = C;
        p.out_f32 = 0;
        p.o_sa = 1;
        p.o_sb = ldc;
        p.a_scale = reinterpret_cast<const __half*>(scale);
        p.res = reinterpret_cast<const __half*>(R);
        p.r_sa = 1;
        p.r_sb = ldr;
    }
    rc = run_gemm(p, w_int8, bt, gx, gy, 1, st);
    if (rc || p.splits == 1) return rc;
    const int64_t total = (int64_t)M * N;
    int blocks = (int)((total + 255) / 256);
    const int cap = num_sms() * 8;
    if (blocks > cap) blocks = cap;
    return launch_pdl(splitk_reduce_kernel, dim3(blocks), dim3(256), 0, st, reinterpret_cast<const float*>(ws), p.splits, M, N,
                                                 reinterpret_cast<const __half*>(scale), alpha,
                                                 reinterpret_cast<const __half*>(R), ldr, reinterpret_cast<__half*>(C),
                                                 ldc);
}

}  // namespace npub

extern "C" int npub_w8a16_gemm(const void* A, int64_t lda, const int8_t* Wq, int64_t ldw, const void* scale, void* C,
                               int64_t ldc, const void* R, int64_t ldr, int M, int N, int K, float alpha,
                               void* workspace, size_t workspace_bytes, void* stream) {
    return npub::linear(true, A, lda, Wq, ldw, scale, C, ldc, R, ldr, M, N, K, alpha, workspace, workspace_bytes,
                        stream);
}

extern "C" size_t npub_w8a16_gemm_workspace(int M, int N, int K) { return npub::linear_workspace(M, N, K, true); }

extern "C" int npub_w8a16_gemm_swiglu(const void* A, int64_t lda, const int8_t* Wq, int64_t ldw, const void* scale,
                                      void* C, int64_t ldc, int M, int F, int K, void* workspace,
                                      size_t workspace_bytes, void* stream) {
    NPUB_CHECK_ARG(M >= 0 && F >= 0 && K >= 0);
    if (M == 0 || F == 0) return NPUB_OK;
    NPUB_CHECK_ARG(A && Wq && C);
    NPUB_CHECK_ARG(K % 16 == 0 && K > 0);
    NPUB_CHECK_ARG(lda >= K && lda % 8 == 0 && npub_aligned(A, 16));
    NPUB_CHECK_ARG(ldw >= K && ldw % 16 == 0 && npub_aligned(Wq, 16));
    NPUB_CHECK_ARG(ldc >= F);
    NPUB_CHECK_ARG(F <= (1 << 29));
    const int N = 2 * F;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (npub::w8a16_use_skinny(M, N, K))
        return npub::w8a16_skinny_run(A, lda, Wq, ldw, scale, C, ldc, nullptr, 0, M, N, K, 1.0f, workspace,
                                      workspace_bytes, st, 1);
    return npub::linear_w8a16_pair(A, lda, Wq, ldw, scale, C, ldc, nullptr, 0, M, N, K, 1.0f, workspace,
                                   workspace_bytes, st, 1);
}

// W8A16 GEMM of a decode step with an RMSNorm folded in (the stream-K
// kernel; M <= 64).  Replaces the pair RMSNorm -> GEMM of the decode layer
// (llama_layer.py:71-152 runs them as separate programs):
//   consumer: A = fp16(h * gamma) of the residual stream h, and row t of the
//     result is scaled by rsqrt(sum_{i < rs_n} rs_part[i rs_ld + t] / rs_d + eps);
//   producer: C = fp16(A Wq^T * scale + R) as npub_w8a16_gemm, plus
//     G = fp16(C * gamma) and the sums of C^2 over every 32 output columns
//     (ss[(n / 32) ss_ld + t]) for the next GEMM to consume;
//   Wq_next (optional): the next W8A16 GEMM of the chain (same M, int8
//     [N_next, K_next]); its first weight tiles are prefetched to L2 once this
//     GEMM's own weights are requested.
extern "C" size_t npub_w8a16_gemm_rms_workspace(int M, int N, int K) {
    return npub::w8a16_skinny_workspace(M, N, K);
}

extern "C" int npub_w8a16_gemm_rms(const void* A, int64_t lda, const int8_t* Wq, int64_t ldw, const void* scale,
                                   void* C, int64_t ldc, const void* R, int64_t ldr, int M, int N, int K, int swiglu,
                                   const float* rs_part, int rs_n, int64_t rs_ld, int rs_d, float rs_eps,
                                   const void* gamma, void* G, int64_t ldg, float* ss, int64_t ss_ld,
                                   const int8_t* Wq_next, int64_t ldw_next, int N_next, int K_next,
                                   void* workspace, size_t workspace_bytes, void* stream) {
    NPUB_CHECK_ARG(M >= 0 && N >= 0 && K >= 0);
    if (M == 0 || N == 0) return NPUB_OK;
    if (!npub::w8a16_skinny_fits(M, N)) return NPUB_ERR_UNSUPPORTED;
    NPUB_CHECK_ARG(A && Wq && C);
    NPUB_CHECK_ARG(K % 16 == 0 && K > 0);
    NPUB_CHECK_ARG(lda >= K && lda % 8 == 0 && npub_aligned(A, 16));
    NPUB_CHECK_ARG(ldw >= K && ldw % 16 == 0 && npub_aligned(Wq, 16));
    NPUB_CHECK_ARG(ldc >= (swiglu ? N / 2 : N));
    NPUB_CHECK_ARG(!swiglu || (N % 2 == 0 && !R && !G && !ss));
    NPUB_CHECK_ARG(!R || ldr >= N);
    NPUB_CHECK_ARG(!rs_part || (rs_n > 0 && rs_ld >= M && rs_d > 0));
    NPUB_CHECK_ARG(!G || (gamma && ldg >= N));
    NPUB_CHECK_ARG(!ss || (N % 32 == 0 && ss_ld >= M));
    npub::SkinnyNorm nrm;
    memset(&nrm, 0, sizeof(nrm));
    nrm.rs_part = rs_part;
    nrm.rs_n = rs_n;
    nrm.rs_ld = rs_ld;
    nrm.rs_d = (float)rs_d;
    nrm.rs_eps = rs_eps;
    nrm.gamma = reinterpret_cast<const __half*>(gamma);
    nrm.G = reinterpret_cast<__half*>(G);
    nrm.ldg = ldg;
    nrm.ss = ss;
    nrm.ss_ld = ss_ld;
    npub::SkinnyNext nx;
    nx.W = Wq_next;
    nx.ldw = ldw_next;
    nx.M = M;
    nx.N = N_next;
    nx.K = K_next;
    return npub::w8a16_skinny_run(A, lda, Wq, ldw, scale, C, ldc, R, ldr, M, N, K, 1.0f, workspace, workspace_bytes,
                                  reinterpret_cast<cudaStream_t>(stream), swiglu ? 1 : 0, &nrm,
                                  Wq_next ? &nx : nullptr);
}

extern "C" const char* npub_w8a16_kernel_name(int M, int N, int K) {
    if (M <= 0 || N <= 0 || K <= 0) return "none";
    if (npub::w8a16_use_skinny(M, N, K)) return "w8a16_skinny_kernel (stream-K, tcgen05 with A in TMEM)";
    return "w8a16_pair_kernel (tcgen05 cta_group::2 W8A16)";
}

extern "C" int npub_f16_gemm(const void* A, int64_t lda, const void* W, int64_t ldw, const void* scale, void* C,
                             int64_t ldc, const void* R, int64_t ldr, int M, int N, int K, float alpha, void* workspace,
                             size_t workspace_bytes, void* stream) {
    return npub::linear(false, A, lda, W, ldw, scale, C, ldc, R, ldr, M, N, K, alpha, workspace, workspace_bytes,
                        stream);
}

extern "C" size_t npub_f16_gemm_workspace(int M, int N, int K) { return npub::linear_workspace(M, N, K, false); }

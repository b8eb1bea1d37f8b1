// Attention for sm_100a.
//
// Prefill (llama_layer.py:114-137, legalize.py:117-127): head_dim 128 runs the
// fused flash-attention kernel of fmha.cu; other head sizes run per head
//   S = Q K^T * scale (tcgen05 GEMM, tiles above the causal diagonal skipped)
//   P = softmax(S) in place (vector_ops.cu)
//   O = P V (tcgen05 GEMM, K loop cut at the diagonal), V transposed once so
//   both GEMM operands are K-major.
// Decode: flash-decoding over an fp16 KV cache [batch, kv_heads, cap, 128],
// HBM-bound: streaming kernels (a bulk-copy ring of K/V stages) for
// grouped-query groups of 1 to 8 heads, scheduled by the number of (sequence,
// kv head) items; larger groups run a split kernel with 4 lanes per key and a
// combine pass.
#include <cstdlib>

#include "common.cuh"
#include "gemm_tc.h"

namespace npub {

int fmha_prefill(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv, void* out,
                 int64_t ldo, int batch, int tokens, int heads, int kv_heads, float scale, int causal,
                 cudaStream_t st);

// V rows of `batch` sequences [batch*T, ldv] (kv head h at columns h*hd) ->
// Vt [batch*kvh, hd, tp] (tokens contiguous, zero past T).
__global__ void transpose_heads_kernel(const __half* __restrict__ v, int64_t ldv, int T, int kvh, int hd,
                                       __half* __restrict__ vt, int64_t tp) {
    __shared__ __half tile[64][64 + 2];
    const int bz = blockIdx.z;  // b * kvh + h
    const int b = bz / kvh, h = bz % kvh;
    const int t0 = blockIdx.x * 64, d0 = blockIdx.y * 64;
    for (int i = threadIdx.y; i < 64; i += blockDim.y) {
        for (int j = threadIdx.x; j < 64; j += blockDim.x) {
            const int t = t0 + i, d = d0 + j;
            tile[i][j] = (t < T && d < hd) ? v[((int64_t)b * T + t) * ldv + (int64_t)h * hd + d] : __float2half(0.0f);
        }
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 64; i += blockDim.y) {
        for (int j = threadIdx.x; j < 64; j += blockDim.x) {
            const int d = d0 + i, t = t0 + j;
            if (d < hd && t < (int)tp) vt[((int64_t)bz * hd + d) * tp + t] = tile[j][i];
        }
    }
}

// ---------------------------------------------------------------- decode
constexpr int kDecHd = 128;
constexpr int kDecWarps = 4;

struct DecodeArgs {
    const __half* q;
    int64_t ldq;
    const __half* kc;
    const __half* vc;
    int64_t cap;
    const int32_t* lens;
    int ctx;
    __half* out;
    int64_t ldo;
    int heads, kv_heads, splits, chunk;
    int batch;
    float scale_log2;  // scale * log2(e)
    float* part;       // split kernel: [bh, splits, hd + 2]; persistent kernel: [CTA, group, hd + 2]
    int* err;          // device error word
    uint64_t wait_ns;  // bound of the finishers' waits
    int tail_first, tail_parts;  // one CTA per item: items >= tail_first run in tail_parts pieces
    int kv_evict_first;          // K/V stage loads marked evict-first in L2 (each key is read once)
};

__device__ __forceinline__ void ld8f(const __half* p, float (&f)[8]) {
    uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 t = __half22float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

// Lane l of a warp: key slot g = l / 4 (8 keys per step), part j = l % 4 owning
// dims {8*(j + 4*i) .. +8 : i = 0..3}, so each 16-byte load instruction of the
// four lanes of a key covers 64 contiguous bytes of the row.
__global__ void __launch_bounds__(kDecWarps * 32) decode_attn_kernel(const DecodeArgs a) {
    const int bh = blockIdx.x;
    const int b = bh / a.heads, h = bh % a.heads;
    const int kvh = h / (a.heads / a.kv_heads);
    const int split = blockIdx.y;
    const int len = min((int64_t)(a.lens ? a.lens[b] : a.ctx), a.cap);
    const int c0 = split * a.chunk;
    const int c1 = min(len, c0 + a.chunk);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, j = lane & 3;

    float q[32];
    const __half* qrow = a.q + (int64_t)b * a.ldq + (int64_t)h * kDecHd;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float f[8];
        ld8f(qrow + 8 * (j + 4 * i), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) q[8 * i + e] = f[e] * a.scale_log2;
    }
    const __half* kbase = a.kc + ((int64_t)b * a.kv_heads + kvh) * a.cap * kDecHd;
    const __half* vbase = a.vc + ((int64_t)b * a.kv_heads + kvh) * a.cap * kDecHd;

    float m = -INFINITY, l = 0.0f, acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.0f;

    // keys handled by this warp: c0 + warp*8 + g, stepping by kDecWarps*8
    for (int key = c0 + warp * 8 + g; key - g < c1; key += kDecWarps * 8) {
        const bool ok = key < c1;
        float kf[32], vf[32];
        const __half* kr = kbase + (int64_t)(ok ? key : c0) * kDecHd;
        const __half* vr = vbase + (int64_t)(ok ? key : c0) * kDecHd;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float f[8];
            ld8f(kr + 8 * (j + 4 * i), f);
#pragma unroll
            for (int e = 0; e < 8; ++e) kf[8 * i + e] = f[e];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float f[8];
            ld8f(vr + 8 * (j + 4 * i), f);
#pragma unroll
            for (int e = 0; e < 8; ++e) vf[8 * i + e] = f[e];
        }
        float sdot = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i) sdot += q[i] * kf[i];
        sdot += __shfl_xor_sync(0xffffffffu, sdot, 1);
        sdot += __shfl_xor_sync(0xffffffffu, sdot, 2);
        if (ok) {
            const float mn = fmaxf(m, sdot);
            const float corr = exp2f(m - mn);
            const float pk = exp2f(sdot - mn);
            l = l * corr + pk;
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[i] = acc[i] * corr + pk * vf[i];
            m = mn;
        }
    }
    // combine the 8 key slots of the warp (lanes with equal j)
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        const float mo = __shfl_xor_sync(0xffffffffu, m, o);
        const float lo = __shfl_xor_sync(0xffffffffu, l, o);
        const float mn = fmaxf(m, mo);
        const float ca = (m == -INFINITY) ? 0.0f : exp2f(m - mn);
        const float cb = (mo == -INFINITY) ? 0.0f : exp2f(mo - mn);
        l = l * ca + lo * cb;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const float ao = __shfl_xor_sync(0xffffffffu, acc[i], o);
            acc[i] = acc[i] * ca + ao * cb;
        }
        m = mn;
    }
    // combine warps through shared memory
    __shared__ float sm_m[kDecWarps], sm_l[kDecWarps];
    __shared__ float sm_acc[kDecWarps][kDecHd];
    if (g == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int e = 0; e < 8; ++e) sm_acc[warp][8 * (j + 4 * i) + e] = acc[8 * i + e];
        if (j == 0) {
            sm_m[warp] = m;
            sm_l[warp] = l;
        }
    }
    __syncthreads();
    if (threadIdx.x < kDecHd) {
        const int d = threadIdx.x;
        float M = -INFINITY;
        for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, sm_m[w]);
        float L = 0.0f, A = 0.0f;
        for (int w = 0; w < kDecWarps; ++w) {
            const float c = (sm_m[w] == -INFINITY) ? 0.0f : exp2f(sm_m[w] - M);
            L += sm_l[w] * c;
            A += sm_acc[w][d] * c;
        }
        if (a.splits == 1) {
            a.out[(int64_t)b * a.ldo + (int64_t)h * kDecHd + d] = __float2half_rn(L > 0.0f ? A / L : 0.0f);
        } else {
            float* pp = a.part + ((int64_t)bh * a.splits + split) * (kDecHd + 2);
            pp[d] = A;
            if (d == 0) {
                pp[kDecHd] = M;
                pp[kDecHd + 1] = L;
            }
        }
    }
}

// Streaming decode attention.  One CTA serves all G = heads / kv_heads query
// heads of a (sequence, kv head) item, so a K/V row is read from HBM once.  K
// and V of 64 consecutive keys are contiguous in the cache ([cap, 128] per
// (sequence, kv head)), so a stage is two 16 KB bulk copies (cp.async.bulk, no
// tensor map) into a 3-deep shared-memory ring, issued by a producer warp;
// with two CTAs per SM ~192 KB of HBM reads are in flight per SM.  Each of the
// eight compute warps owns 8 keys of every stage and keeps its own online
// softmax (no block barrier per stage):
//   scores: a half-warp per key, 16 lanes x 8 dims, four shuffles;
//   P V:    lane l accumulates dims [4 l, 4 l + 4) of every query head;
// the warps release a stage through an mbarrier and merge through shared
// memory at the end of an item.  Two schedules share that stage code:
//  * many items (batch x heads >= 6 x SMs): one CTA per item, the hardware
//    handing items to SMs as CTAs finish;
//  * few items: a persistent grid (as many CTAs as are resident at once) over
//    the list of 64-key stages of all items, sequence-major; CTA c takes
//    stages [c S / G, (c + 1) S / G) of the S, so every SM streams the same
//    number of K/V bytes whatever the batch and lengths are, and the producer
//    runs on across item boundaries (the first stage of an item in a CTA also
//    brings the item's query rows).  An item cut between CTAs is finished by
//    the CTA holding its first stage (its last piece); the CTAs holding the
//    other pieces do them first (each such piece starts their range), publish
//    (acc, max, sum) per head and set a flag, and the finisher merges them in
//    CTA order, so the result does not depend on timing.  Only finishers
//    wait, only on pieces other CTAs do first, and every CTA is resident, so
//    no wait can close a cycle.  This replaces the split-context kernel and
//    its combine pass (measured 4-14 % faster where that needed splits).
constexpr int kStKeys = 64;
constexpr int kStBytes = kStKeys * kDecHd * 2;  // one of K or V per stage
// K/V ring depth NS (a template argument): 2 or 3 stages, chosen per call.
constexpr int kStWarps = 8;                     // compute warps; warp 8 is the producer
constexpr int kStKeysPerWarp = kStKeys / kStWarps;  // 8: four pairs of keys per stage
constexpr int kStThreads = (kStWarps + 1) * 32;
constexpr int kPsMaxSeq = 512;   // sequences whose stage prefix sums fit in shared memory
constexpr int kPsMaxCtas = 1024;

// One flag per CTA slot of the persistent kernel: set when the CTA's first
// piece (of an item started by an earlier CTA) is published, cleared by the
// item's finisher, so every completed call leaves them zero.
__device__ uint32_t g_decode_piece_flag[kPsMaxCtas];
// Pieces of the split tail items of the one-CTA-per-item schedule that have
// arrived (the last one merges them and clears the count).
__device__ int g_decode_tail_cnt[kPsMaxCtas];
constexpr int kTailPartsMax = 4;

// NPUB_DECODE_TAIL_SPLIT=0 keeps every item in one CTA.
static bool tail_split_enabled() {
    static const int on = [] {
        const char* v = getenv("NPUB_DECODE_TAIL_SPLIT");
        return v && v[0] == '0' ? 0 : 1;
    }();
    return on != 0;
}

template <int G, int NS>
constexpr int stream_smem() {
    return NS * 2 * kStBytes + 16 * NS + 128;
}

template <int G, int NS>
struct PsLayout {
    static constexpr int kQ = G * kDecHd * 2;  // query rows of one item
    static constexpr int kQOff = NS * 2 * kStBytes;
    static constexpr int kMergeOff = kQOff + NS * kQ;
    static constexpr int kPreOff = kMergeOff + kStWarps * (kDecHd + 2) * 4;
    static constexpr int kLenOff = kPreOff + (kPsMaxSeq + 1) * 4;
    static constexpr int kBarOff = (kLenOff + kPsMaxSeq * 4 + 7) / 8 * 8;
    static constexpr int kAbortOff = kBarOff + 2 * NS * 8;
    static constexpr int kTotal = kAbortOff + 16 + 128;  // + 128: base alignment
};

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// bulk_load with an L2 cache policy.
__device__ __forceinline__ void bulk_load_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

// L2 prefetch of the first stages of a (sequence, kv head)'s keys [k0, k1),
// issued before griddepcontrol.wait: only the newest key is written by the
// kernels this one follows, and L2 stays coherent with that write.
__device__ __forceinline__ void prefetch_kv_l2(const DecodeArgs& a, int b, int kvh, int64_t k0, int64_t k1) {
    if (k1 <= k0) return;
    const int64_t off = (((int64_t)b * a.kv_heads + kvh) * a.cap + k0) * kDecHd;
    const uint32_t bytes = (uint32_t)(k1 - k0) * kDecHd * 2;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.kc + off), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.vc + off), "r"(bytes) : "memory");
}

// Barrier of the eight compute warps (the producer warp has left); the
// non-.aligned form, since lane 0 of warp 0 may arrive from a finisher's wait.
__device__ __forceinline__ void compute_bar() { asm volatile("barrier.sync 1, %0;" ::"n"(kStWarps * 32) : "memory"); }

__device__ __forceinline__ void st_cg_f32(float* p, float v) {
    asm volatile("st.global.cg.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

// One 64-key stage (n valid keys): the warp's 8 keys scored against its G
// query heads (q pre-scaled by scale * log2 e), online softmax, P V into the
// lane's 4 dims.
template <int G>
__device__ __forceinline__ void stream_stage(const uint8_t* Ks, const uint8_t* Vs, int n, int warp, int lane,
                                             const float (&q)[G][8], float (&m)[G], float (&l)[G],
                                             float (&acc)[G][4]) {
    const int hw = lane >> 4, l16 = lane & 15;
    constexpr int NP = kStKeysPerWarp / 2;
    // scores of keys kStKeysPerWarp warp + 2 it + hw
    float sc[G][NP];
#pragma unroll
    for (int it = 0; it < NP; ++it) {
        const int key = kStKeysPerWarp * warp + 2 * it + hw;
        const uint4 raw = *reinterpret_cast<const uint4*>(Ks + key * (kDecHd * 2) + l16 * 16);
        const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
        float kf[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 t = __half22float2(h2[e]);
            kf[2 * e] = t.x;
            kf[2 * e + 1] = t.y;
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float x = 0.0f;
#pragma unroll
            for (int e = 0; e < 8; ++e) x = fmaf(q[g][e], kf[e], x);
            x += __shfl_xor_sync(0xffffffffu, x, 8);
            x += __shfl_xor_sync(0xffffffffu, x, 4);
            x += __shfl_xor_sync(0xffffffffu, x, 2);
            x += __shfl_xor_sync(0xffffffffu, x, 1);
            sc[g][it] = key < n ? x : -INFINITY;
        }
    }
    // online softmax over this warp's keys
    float p[G][NP];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        float mx = sc[g][0];
#pragma unroll
        for (int it = 1; it < NP; ++it) mx = fmaxf(mx, sc[g][it]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float mn = fmaxf(m[g], mx);
        const float corr = (m[g] == -INFINITY) ? 0.0f : exp2f(m[g] - mn);
        float sum = 0.0f;
#pragma unroll
        for (int it = 0; it < NP; ++it) {
            p[g][it] = sc[g][it] == -INFINITY ? 0.0f : exp2f(sc[g][it] - mn);
            sum += p[g][it];
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 16);
        l[g] = l[g] * corr + sum;
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[g][e] *= corr;
        m[g] = mn == -INFINITY ? m[g] : mn;
    }
    // P V: lane owns dims 4 lane .. 4 lane + 3
#pragma unroll
    for (int it = 0; it < NP; ++it) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int key = kStKeysPerWarp * warp + 2 * it + hh;
            if (key < n) {  // warp-uniform; rows past n may hold stale bytes
                const uint2 raw = *reinterpret_cast<const uint2*>(Vs + key * (kDecHd * 2) + lane * 8);
                const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
                const float2 v01 = __half22float2(h2[0]), v23 = __half22float2(h2[1]);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float pk = __shfl_sync(0xffffffffu, p[g][it], hh * 16);
                    acc[g][0] = fmaf(pk, v01.x, acc[g][0]);
                    acc[g][1] = fmaf(pk, v01.y, acc[g][1]);
                    acc[g][2] = fmaf(pk, v23.x, acc[g][2]);
                    acc[g][3] = fmaf(pk, v23.y, acc[g][3]);
                }
            }
        }
    }
}

// ------------------------------------------------ one CTA per (sequence, kv head)
template <int G, int NS>
__global__ void __launch_bounds__(kStThreads, G <= 4 ? 2 : 1) decode_attn_stream_kernel(const DecodeArgs a) {
    pdl_trigger();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + NS * 2 * kStBytes);
    uint64_t* empty = full + NS;
    static_assert(kStWarps * G * (kDecHd + 2) * 4 <= NS * 2 * kStBytes, "merge area reuses the ring");

    // item = sequence * kv_heads + kv head; the items of the last, partial
    // wave (>= tail_first) run in tail_parts pieces of whole 64-key stages
    int item = blockIdx.x, part = 0, parts = 1;
    if (a.tail_parts > 1 && (int)blockIdx.x >= a.tail_first) {
        const int t = (int)blockIdx.x - a.tail_first;
        item = a.tail_first + t / a.tail_parts;
        part = t % a.tail_parts;
        parts = a.tail_parts;
    }
    const int b = item / a.kv_heads, kvh = item % a.kv_heads;
    const int split = blockIdx.y;  // context split (a.splits > 1: partials for decode_combine_kernel)
    if (threadIdx.x == kStWarps * 32) {
        int64_t k0 = (int64_t)split * a.chunk;
        if (parts > 1) {  // the guess: every length is the largest (ctx)
            const int64_t n = (min((int64_t)a.ctx, a.cap) + kStKeys - 1) / kStKeys;
            k0 = part * n / parts * kStKeys;
        }
        prefetch_kv_l2(a, b, kvh, k0, min(min(k0 + NS * kStKeys, k0 + (int64_t)a.chunk), a.cap));
    }
    pdl_wait();  // lens, q and the caches come from earlier kernels
    const int len = (int)min((int64_t)(a.lens ? a.lens[b] : a.ctx), a.cap);
    int c0 = split * a.chunk;
    int c1 = min(len, c0 + a.chunk);
    if (parts > 1) {
        const int n = (len + kStKeys - 1) / kStKeys;
        c0 = part * n / parts * kStKeys;
        c1 = min(len, (part + 1) * n / parts * kStKeys);
    }
    const int nkeys = c1 > c0 ? c1 - c0 : 0;
    const int nst = (nkeys + kStKeys - 1) / kStKeys;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kStWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();
    int never = 0;
    volatile int* no_abort = &never;

    float m[G], l[G], acc[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[g][e] = 0.0f;
    }

    if (warp == kStWarps) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const __half* kbase = a.kc + (((int64_t)b * a.kv_heads + kvh) * a.cap + c0) * kDecHd;
            const __half* vbase = a.vc + (((int64_t)b * a.kv_heads + kvh) * a.cap + c0) * kDecHd;
            const uint64_t pol = l2_evict_first_policy();
            int i = 0;
            for (; i < nst; ++i) {
                const int slot = i % NS;
                if (i >= NS &&
                    !mbar_wait_bounded(&empty[slot], ((uint32_t)(i / NS) & 1u) ^ 1u, no_abort)) {
                    if (a.err) atomicCAS(a.err, 0, 0x401);
                    break;
                }
                const int k0 = i * kStKeys;
                const uint32_t bytes = (uint32_t)min(kStKeys, nkeys - k0) * kDecHd * 2;
                mbar_arrive_expect_tx(&full[slot], 2 * bytes);
                if (a.kv_evict_first) {
                    bulk_load_hint(ring + slot * 2 * kStBytes, kbase + (int64_t)k0 * kDecHd, bytes, &full[slot], pol);
                    bulk_load_hint(ring + slot * 2 * kStBytes + kStBytes, vbase + (int64_t)k0 * kDecHd, bytes,
                                   &full[slot], pol);
                } else {
                    bulk_load(ring + slot * 2 * kStBytes, kbase + (int64_t)k0 * kDecHd, bytes, &full[slot]);
                    bulk_load(ring + slot * 2 * kStBytes + kStBytes, vbase + (int64_t)k0 * kDecHd, bytes, &full[slot]);
                }
            }
            // every copy issued has landed before the ring is reused or the CTA exits
            for (int j = i - NS < 0 ? 0 : i - NS; j < i; ++j)
                if (!mbar_wait_bounded(&full[j % NS], (uint32_t)(j / NS) & 1u, no_abort, 200000000ull) &&
                    a.err)
                    atomicCAS(a.err, 0, 0x402);
        }
    } else {
        // ------------------------------------------------------------ compute warps
        const int l16 = lane & 15;
        float q[G][8];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float f[8];
            ld8f(a.q + (int64_t)b * a.ldq + (int64_t)(kvh * G + g) * kDecHd + 8 * l16, f);
#pragma unroll
            for (int e = 0; e < 8; ++e) q[g][e] = f[e] * a.scale_log2;
        }
        for (int i = 0; i < nst; ++i) {
            const int slot = i % NS;
            const bool ok = mbar_wait_bounded(&full[slot], (uint32_t)(i / NS) & 1u, no_abort);
            if (!__all_sync(0xffffffffu, ok)) {
                if (lane == 0 && a.err) atomicCAS(a.err, 0, 0x403);
                break;
            }
            const uint8_t* Ks = ring + slot * 2 * kStBytes;
            stream_stage<G>(Ks, Ks + kStBytes, min(kStKeys, nkeys - i * kStKeys), warp, lane, q, m, l, acc);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
    }
    // merge the compute warps (the ring is idle now: every copy has landed and
    // been read); only lane 0 of the producer warp ran the copy loop, hence the
    // thread-counting barrier
    cta_sync_divergent();
    float* mg = reinterpret_cast<float*>(ring);  // [warp][g][130]: acc[128], m, l
    if (warp < kStWarps) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float* row = mg + (warp * G + g) * (kDecHd + 2);
#pragma unroll
            for (int e = 0; e < 4; ++e) row[4 * lane + e] = acc[g][e];
            if (lane == 0) {
                row[kDecHd] = m[g];
                row[kDecHd + 1] = l[g];
            }
        }
    }
    __syncthreads();
    if (threadIdx.x < kDecHd) {
        const int d = threadIdx.x;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float M = -INFINITY;
            for (int w = 0; w < kStWarps; ++w) M = fmaxf(M, mg[(w * G + g) * (kDecHd + 2) + kDecHd]);
            float L = 0.0f, A = 0.0f;
            for (int w = 0; w < kStWarps; ++w) {
                const float* row = mg + (w * G + g) * (kDecHd + 2);
                const float c = row[kDecHd] == -INFINITY ? 0.0f : exp2f(row[kDecHd] - M);
                L += row[kDecHd + 1] * c;
                A += row[d] * c;
            }
            const int h = kvh * G + g;
            if (parts > 1) {
                // this piece's (acc, m, l) for the item's last piece to merge
                float* pp = a.part + ((int64_t)((int)blockIdx.x - a.tail_first) * G + g) * (kDecHd + 2);
                pp[d] = A;
                if (d == 0) {
                    pp[kDecHd] = M;
                    pp[kDecHd + 1] = L;
                }
            } else if (a.splits == 1) {
                a.out[(int64_t)b * a.ldo + (int64_t)h * kDecHd + d] = __float2half_rn(L > 0.0f ? A / L : 0.0f);
            } else {
                float* pp = a.part + (((int64_t)b * a.heads + h) * a.splits + split) * (kDecHd + 2);
                pp[d] = A;
                if (d == 0) {
                    pp[kDecHd] = M;
                    pp[kDecHd + 1] = L;
                }
            }
        }
    }
    if (parts == 1) return;
    // ---------------------------------------------------- tail item: last piece merges
    __shared__ int last_piece;
    const int ti = (item - a.tail_first);  // tail item index
    __threadfence();                        // this piece's rows before its arrival
    __syncthreads();
    if (threadIdx.x == 0) {
        const int seen = atomicAdd(&g_decode_tail_cnt[ti], 1);
        last_piece = seen == parts - 1;
        if (last_piece) g_decode_tail_cnt[ti] = 0;  // every piece of the item has arrived
        __threadfence();
    }
    __syncthreads();
    if (!last_piece || threadIdx.x >= kDecHd) return;
    const int d = threadIdx.x;
    const float* base = a.part + (int64_t)ti * parts * G * (kDecHd + 2);
#pragma unroll
    for (int g = 0; g < G; ++g) {
        // pieces in part order, whichever arrived last: the same sums every run
        float M = -INFINITY;
        for (int p = 0; p < parts; ++p) M = fmaxf(M, __ldcg(base + (p * G + g) * (kDecHd + 2) + kDecHd));
        float L = 0.0f, A = 0.0f;
        for (int p = 0; p < parts; ++p) {
            const float* row = base + (p * G + g) * (kDecHd + 2);
            const float mp = __ldcg(row + kDecHd);
            const float c = mp == -INFINITY ? 0.0f : exp2f(mp - M);
            L += __ldcg(row + kDecHd + 1) * c;
            A += __ldcg(row + d) * c;
        }
        a.out[(int64_t)b * a.ldo + (int64_t)(kvh * G + g) * kDecHd + d] =
            __float2half_rn(L > 0.0f ? A / L : 0.0f);
    }
}

template <int G, int NS>
static int launch_stream(DecodeArgs a, int batch, int kv_heads, int splits, void* workspace, size_t workspace_bytes,
                         cudaStream_t st) {
    auto kern = decode_attn_stream_kernel<G, NS>;
    constexpr int smem = stream_smem<G, NS>();
    static int occ = 0;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess && occ == 0) {
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kStThreads, smem);
        if (e == cudaSuccess && occ <= 0) occ = 1;
    }
    if (e != cudaSuccess) {
        occ = 0;
        npub_internal_set_cuda_error(e);
        return NPUB_ERR_CUDA;
    }
    // The items past the last whole wave of resident CTAs would run alone, each
    // CTA's stream bound by its ring's latency: run them in pieces that fill
    // the idle slots and let each item's last piece merge them.
    const int items = batch * kv_heads;
    const int slots = num_sms() * occ;
    const int tail = items > slots ? items % slots : 0;
    const int stages = (int)((max(a.ctx, 1) + kStKeys - 1) / kStKeys);
    int parts = tail > 0 ? min(kTailPartsMax, slots / tail) : 1;
    parts = min(parts, stages / 2);
    a.tail_first = items - tail;
    a.tail_parts = 1;
    int grid = items;
    if (splits == 1 && parts >= 2 && tail <= kPsMaxCtas && workspace &&
        (size_t)tail * parts * G * (kDecHd + 2) * sizeof(float) <= workspace_bytes && tail_split_enabled()) {
        a.tail_parts = parts;
        a.part = reinterpret_cast<float*>(workspace);
        grid = items - tail + tail * parts;
    }
    return launch_pdl(kern, dim3(grid, splits), dim3(kStThreads), smem, st, a);
}

// ------------------------------------------------ persistent grid over the stage list
// Position in the stage list: sequence b, kv head h, stage s of the item's n.
struct PsCursor {
    int b, h, s, n;
};

// pre[b] = kv_heads * (stages of sequences < b); f < pre[batch].
__device__ __forceinline__ PsCursor ps_locate(int f, const int* pre, int batch, int kvh) {
    int lo = 0, hi = batch - 1;  // the last b with pre[b] <= f (its item count is non-zero)
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (pre[mid] <= f) lo = mid;
        else hi = mid - 1;
    }
    PsCursor c;
    c.b = lo;
    c.n = (pre[lo + 1] - pre[lo]) / kvh;
    const int off = f - pre[lo];
    c.h = off / c.n;
    c.s = off - c.h * c.n;
    return c;
}

__device__ __forceinline__ void ps_advance(PsCursor& c, const int* pre, int batch, int kvh) {
    if (++c.s < c.n) return;
    c.s = 0;
    if (++c.h < kvh) return;
    c.h = 0;
    do {
        ++c.b;
    } while (c.b < batch && pre[c.b + 1] == pre[c.b]);
    if (c.b < batch) c.n = (pre[c.b + 1] - pre[c.b]) / kvh;
}

// CTA cc of nctas has no stages (more CTAs than stages): it publishes nothing.
__device__ __forceinline__ bool ps_empty(int cc, int S, int nctas) {
    return (int64_t)cc * S / nctas == (int64_t)(cc + 1) * S / nctas;
}

template <int G, int NS>
__global__ void __launch_bounds__(kStThreads, G > 4 ? 1 : 2) decode_attn_persist_kernel(const DecodeArgs a) {
    using L = PsLayout<G, NS>;
    pdl_trigger();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    uint8_t* ring = base;
    const uint8_t* qarea = base + L::kQOff;
    float* mg = reinterpret_cast<float*>(base + L::kMergeOff);  // [warp][130]: acc[128], m, l of one head
    int* pre = reinterpret_cast<int*>(base + L::kPreOff);
    int* lens = reinterpret_cast<int*>(base + L::kLenOff);
    uint64_t* full = reinterpret_cast<uint64_t*>(base + L::kBarOff);
    uint64_t* empty = full + NS;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(base + L::kAbortOff);
    static_assert(L::kTotal <= 227 * 1024, "shared memory budget");

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int batch = a.batch, kvh = a.kv_heads;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kStWarps);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (threadIdx.x == kStWarps * 32 && a.ctx > 0) {
        // the first stages of this CTA's range if every length is the largest
        // (ctx): the usual case, and only a prefetch when it is not
        const int64_t n = (min((int64_t)a.ctx, a.cap) + kStKeys - 1) / kStKeys;
        const int64_t S = (int64_t)batch * kvh * n;
        int64_t f = (int64_t)blockIdx.x * S / gridDim.x;
        const int64_t fe = min(f + NS, ((int64_t)blockIdx.x + 1) * S / gridDim.x);
        while (f < fe) {
            const int64_t item = f / n, st = f % n;
            const int64_t k0 = st * kStKeys, k1 = min(min((int64_t)a.ctx, a.cap), k0 + (fe - f) * kStKeys);
            const int64_t kend = min(k1, n * kStKeys);
            prefetch_kv_l2(a, (int)(item / kvh), (int)(item % kvh), k0, min(kend, min((int64_t)a.ctx, a.cap)));
            f += (kend - k0 + kStKeys - 1) / kStKeys;
        }
    }
    pdl_wait();  // lens, q and the caches come from earlier kernels
    if (warp == 0) {
        int carry = 0;
        for (int b0 = 0; b0 < batch; b0 += 32) {
            const int b = b0 + lane;
            int n = 0;
            if (b < batch) {
                int64_t len = a.lens ? (int64_t)a.lens[b] : (int64_t)a.ctx;
                len = len < 0 ? 0 : (len > a.cap ? a.cap : len);
                lens[b] = (int)len;
                n = (int)((len + kStKeys - 1) / kStKeys) * kvh;
            }
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, n, o);
                if (lane >= o) n += y;
            }
            if (b < batch) pre[b + 1] = carry + n;
            carry += __shfl_sync(0xffffffffu, n, 31);
        }
        if (lane == 0) pre[0] = 0;
    }
    __syncthreads();
    const int S = pre[batch];
    const int c = blockIdx.x, nctas = gridDim.x;
    const int f0 = (int)((int64_t)c * S / nctas), f1 = (int)((int64_t)(c + 1) * S / nctas);
    const bool any_empty = S < nctas;  // else every CTA has at least one stage

    if (warp == kStWarps) {
        // ------------------------------------------------------------ producer
        if (lane == 0 && f0 < f1) {
            PsCursor cu = ps_locate(f0, pre, batch, kvh);
            const uint64_t pol = l2_evict_first_policy();
            int i = 0;
            for (int f = f0; f < f1; ++f, ++i) {
                const int slot = i % NS;
                if (i >= NS &&
                    !mbar_wait_bounded(&empty[slot], ((uint32_t)(i / NS) & 1u) ^ 1u, abort_flag)) {
                    if (a.err) atomicCAS(a.err, 0, 0x401);
                    break;
                }
                const bool qload = i == 0 || cu.s == 0;
                const int k0 = cu.s * kStKeys;
                const uint32_t bytes = (uint32_t)min(kStKeys, lens[cu.b] - k0) * kDecHd * 2;
                const int64_t kv = (((int64_t)cu.b * kvh + cu.h) * a.cap + k0) * kDecHd;
                mbar_arrive_expect_tx(&full[slot], 2 * bytes + (qload ? (uint32_t)L::kQ : 0u));
                if (a.kv_evict_first) {
                    bulk_load_hint(ring + slot * 2 * kStBytes, a.kc + kv, bytes, &full[slot], pol);
                    bulk_load_hint(ring + slot * 2 * kStBytes + kStBytes, a.vc + kv, bytes, &full[slot], pol);
                } else {
                    bulk_load(ring + slot * 2 * kStBytes, a.kc + kv, bytes, &full[slot]);
                    bulk_load(ring + slot * 2 * kStBytes + kStBytes, a.vc + kv, bytes, &full[slot]);
                }
                if (qload)
                    bulk_load(base + L::kQOff + slot * L::kQ, a.q + (int64_t)cu.b * a.ldq + (int64_t)cu.h * G * kDecHd,
                              (uint32_t)L::kQ, &full[slot]);
                ps_advance(cu, pre, batch, kvh);
            }
            // every copy issued has landed before the ring is reused or the CTA exits
            int never = 0;
            for (int j = i - NS < 0 ? 0 : i - NS; j < i; ++j)
                if (!mbar_wait_bounded(&full[j % NS], (uint32_t)(j / NS) & 1u, &never, 200000000ull) &&
                    a.err)
                    atomicCAS(a.err, 0, 0x402);
        }
        return;
    }

    // ---------------------------------------------------------------- compute warps
    const int ct = threadIdx.x;  // 0 .. 255
    const int l16 = lane & 15;
    float q[G][8], m[G], l[G], acc[G][4];
    if (f0 < f1) {
        PsCursor cu = ps_locate(f0, pre, batch, kvh);
        for (int f = f0, i = 0; f < f1; ++f, ++i) {
            const int slot = i % NS;
            const bool good =
                __all_sync(0xffffffffu, mbar_wait_bounded(&full[slot], (uint32_t)(i / NS) & 1u, abort_flag));
            if (!good && lane == 0) {
                if (a.err) atomicCAS(a.err, 0, 0x403);
                *abort_flag = 1;
            }
            const uint8_t* Ks = ring + slot * 2 * kStBytes;
            const uint8_t* Vs = Ks + kStBytes;
            if (i == 0 || cu.s == 0) {
                // a new piece: the item's query rows came with this stage
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    m[g] = -INFINITY;
                    l[g] = 0.0f;
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[g][e] = 0.0f;
                    const uint4 raw =
                        good ? *reinterpret_cast<const uint4*>(qarea + slot * L::kQ + g * kDecHd * 2 + l16 * 16)
                             : make_uint4(0, 0, 0, 0);
                    const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 t = __half22float2(h2[e]);
                        q[g][2 * e] = t.x * a.scale_log2;
                        q[g][2 * e + 1] = t.y * a.scale_log2;
                    }
                }
            }
            if (good) stream_stage<G>(Ks, Vs, min(kStKeys, lens[cu.b] - cu.s * kStKeys), warp, lane, q, m, l, acc);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);

            if (cu.s == cu.n - 1 || f == f1 - 1) {
                // ---------------------------------------- end of this CTA's piece of the item
                // (every compute warp takes this branch at the same stage)
                const int is = pre[cu.b] + cu.h * cu.n, ie = is + cu.n;
                const bool has_first = is >= f0, has_last = ie <= f1;
                const int c_last = has_last ? c : (int)(((int64_t)ie * nctas - 1) / S);  // owner of stage ie - 1
                if (has_first && !has_last) {
                    // the finisher: the later pieces were each their CTA's first
                    // work; their flags are polled by all compute threads at once
                    const uint64_t t0 = globaltimer_ns();
                    for (int cc = c + 1 + ct; cc <= c_last; cc += kStWarps * 32) {
                        if (any_empty && ps_empty(cc, S, nctas)) continue;
                        uint32_t it = 0;
                        while (ld_acquire_gpu(&g_decode_piece_flag[cc]) == 0u) {
                            if ((++it & 255u) == 0 && (*abort_flag || globaltimer_ns() - t0 > a.wait_ns)) {
                                if (a.err) atomicCAS(a.err, 0, 0x405);
                                *abort_flag = 1;
                                break;
                            }
                        }
                        if (*abort_flag) break;
                    }
                    __threadfence();
                }
                // the warps' partial softmax states, merged per head through
                // shared memory (threads 0..127: one head dimension each)
                float oM[G], oL[G], oA[G];
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float* row = mg + warp * (kDecHd + 2);
#pragma unroll
                    for (int e = 0; e < 4; ++e) row[4 * lane + e] = acc[g][e];
                    if (lane == 0) {
                        row[kDecHd] = m[g];
                        row[kDecHd + 1] = l[g];
                    }
                    compute_bar();
                    oM[g] = -INFINITY;
                    oL[g] = oA[g] = 0.0f;
                    if (ct < kDecHd) {
#pragma unroll
                        for (int w = 0; w < kStWarps; ++w) oM[g] = fmaxf(oM[g], mg[w * (kDecHd + 2) + kDecHd]);
#pragma unroll
                        for (int w = 0; w < kStWarps; ++w) {
                            const float* r = mg + w * (kDecHd + 2);
                            const float cf = r[kDecHd] == -INFINITY ? 0.0f : exp2f(r[kDecHd] - oM[g]);
                            oL[g] += r[kDecHd + 1] * cf;
                            oA[g] += r[ct] * cf;
                        }
                    }
                    compute_bar();
                }
                if (!has_first) {
                    // a later piece: publish (acc, max, sum) per head, then the flag
                    if (ct < kDecHd) {
#pragma unroll
                        for (int g = 0; g < G; ++g) {
                            float* pp = a.part + ((int64_t)c * G + g) * (kDecHd + 2);
                            st_cg_f32(pp + ct, oA[g]);
                            if (ct == 0) {
                                st_cg_f32(pp + kDecHd, oM[g]);
                                st_cg_f32(pp + kDecHd + 1, oL[g]);
                            }
                        }
                    }
                    __threadfence();
                    compute_bar();
                    if (ct == 0) atomicExch(&g_decode_piece_flag[c], 1u);
                } else {
                    if (!has_last) {
                        // the finisher (this was the CTA's last stage, so the ring is
                        // idle): the later pieces are copied into it in chunks by all
                        // compute threads, then merged in CTA order
                        float* stg = reinterpret_cast<float*>(ring);
                        constexpr int kPiece = G * (kDecHd + 2);
                        constexpr int kChunk = NS * 2 * kStBytes / (kPiece * 4);
                        static_assert(kPiece % 2 == 0, "pieces are copied as float2");
                        for (int cc0 = c + 1; cc0 <= c_last; cc0 += kChunk) {
                            const int np = min(kChunk, c_last - cc0 + 1);
                            // 8-byte loads, eight in flight per thread (kPiece is even and
                            // the workspace 256-byte aligned)
                            const float2* src = reinterpret_cast<const float2*>(a.part + (int64_t)cc0 * kPiece);
                            float2* dst = reinterpret_cast<float2*>(stg);
                            const int n2 = np * kPiece / 2;
                            for (int x0 = ct; x0 < n2; x0 += 8 * kStWarps * 32) {
                                float2 v[8];
#pragma unroll
                                for (int u = 0; u < 8; ++u) {
                                    const int x = x0 + u * kStWarps * 32;
                                    v[u] = x < n2 ? __ldcg(src + x) : make_float2(0.0f, 0.0f);
                                }
#pragma unroll
                                for (int u = 0; u < 8; ++u) {
                                    const int x = x0 + u * kStWarps * 32;
                                    if (x < n2) dst[x] = v[u];
                                }
                            }
                            if (any_empty) {
                                // CTAs without stages published nothing: neutral pieces
                                __syncwarp();
                                compute_bar();
                                for (int x = ct; x < np * kPiece; x += kStWarps * 32)
                                    if (ps_empty(cc0 + x / kPiece, S, nctas))
                                        stg[x] = (x % (kDecHd + 2)) == kDecHd ? -INFINITY : 0.0f;
                            }
                            compute_bar();
                            if (ct < kDecHd) {
                                for (int pc = 0; pc < np; ++pc) {
#pragma unroll
                                    for (int g = 0; g < G; ++g) {
                                        const float* r = stg + pc * kPiece + g * (kDecHd + 2);
                                        const float mo = r[kDecHd];
                                        const float Mn = fmaxf(oM[g], mo);
                                        if (Mn == -INFINITY) continue;
                                        const float c0 = oM[g] == -INFINITY ? 0.0f : exp2f(oM[g] - Mn);
                                        const float c1 = mo == -INFINITY ? 0.0f : exp2f(mo - Mn);
                                        oL[g] = oL[g] * c0 + r[kDecHd + 1] * c1;
                                        oA[g] = oA[g] * c0 + r[ct] * c1;
                                        oM[g] = Mn;
                                    }
                                }
                            }
                            compute_bar();
                        }
                        if (ct == 0)
                            for (int cc = c + 1; cc <= c_last; ++cc) g_decode_piece_flag[cc] = 0u;  // left zero
                    }
                    if (ct < kDecHd) {
#pragma unroll
                        for (int g = 0; g < G; ++g)
                            a.out[(int64_t)cu.b * a.ldo + (int64_t)(cu.h * G + g) * kDecHd + ct] =
                                __float2half_rn(oL[g] > 0.0f ? oA[g] / oL[g] : 0.0f);
                    }
                }
            }
            ps_advance(cu, pre, batch, kvh);
        }
    }
    // sequences without keys: rows of zeros
    for (int b = c; b < batch; b += nctas)
        if (lens[b] == 0)
            for (int x = ct; x < a.heads * kDecHd; x += kStWarps * 32)
                a.out[(int64_t)b * a.ldo + x] = __float2half_rn(0.0f);
}

template <int G, int NS>
static int ps_occupancy() {
    static int occ = 0;
    if (occ == 0) {
        int o = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, decode_attn_persist_kernel<G, NS>, kStThreads,
                                                          PsLayout<G, NS>::kTotal) != cudaSuccess ||
            o <= 0) {
            cudaGetLastError();
            o = 1;
        }
        occ = o;
    }
    return occ;
}

// Grid: every CTA resident at once (the finishers wait on other CTAs), and at
// least ~4 stages per CTA.
static int ps_max_ctas() { return min(kPsMaxCtas, num_sms() * 2); }

template <int G, int NS>
static int launch_persist(DecodeArgs a, int64_t stages_max, size_t workspace_bytes, cudaStream_t st) {
    auto kern = decode_attn_persist_kernel<G, NS>;
    constexpr int smem = PsLayout<G, NS>::kTotal;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
        npub_internal_set_cuda_error(e);
        return NPUB_ERR_CUDA;
    }
    int64_t grid = (int64_t)num_sms() * ps_occupancy<G, NS>();
    grid = min(grid, (int64_t)ps_max_ctas());
    grid = min(grid, max((int64_t)1, (stages_max + 3) / 4));
    if ((size_t)grid * G * (kDecHd + 2) * sizeof(float) > workspace_bytes || !a.part) return NPUB_ERR_WORKSPACE;
    return launch_pdl(kern, dim3((unsigned)grid), dim3(kStThreads), smem, st, a);
}

template <int NS>
static int stream_by_group(int group, const DecodeArgs& a, int batch, int kv_heads, int splits, void* ws,
                           size_t ws_bytes, cudaStream_t st) {
    switch (group) {
        case 1: return launch_stream<1, NS>(a, batch, kv_heads, splits, ws, ws_bytes, st);
        case 2: return launch_stream<2, NS>(a, batch, kv_heads, splits, ws, ws_bytes, st);
        case 3: return launch_stream<3, NS>(a, batch, kv_heads, splits, ws, ws_bytes, st);
        case 4: return launch_stream<4, NS>(a, batch, kv_heads, splits, ws, ws_bytes, st);
        case 5: return launch_stream<5, NS>(a, batch, kv_heads, splits, ws, ws_bytes, st);
        case 6: return launch_stream<6, NS>(a, batch, kv_heads, splits, ws, ws_bytes, st);
        case 7: return launch_stream<7, NS>(a, batch, kv_heads, splits, ws, ws_bytes, st);
        default: return launch_stream<8, NS>(a, batch, kv_heads, splits, ws, ws_bytes, st);
    }
}

template <int NS>
static int persist_by_group(int group, const DecodeArgs& a, int64_t stages, size_t workspace_bytes,
                            cudaStream_t st) {
    switch (group) {
        case 1: return launch_persist<1, NS>(a, stages, workspace_bytes, st);
        case 2: return launch_persist<2, NS>(a, stages, workspace_bytes, st);
        case 3: return launch_persist<3, NS>(a, stages, workspace_bytes, st);
        case 4: return launch_persist<4, NS>(a, stages, workspace_bytes, st);
        case 5: return launch_persist<5, NS>(a, stages, workspace_bytes, st);
        case 6: return launch_persist<6, NS>(a, stages, workspace_bytes, st);
        case 7: return launch_persist<7, NS>(a, stages, workspace_bytes, st);
        default: return launch_persist<8, NS>(a, stages, workspace_bytes, st);
    }
}

__global__ void decode_combine_kernel(const float* __restrict__ part, int splits, int heads, __half* __restrict__ out,
                                      int64_t ldo) {
    pdl_trigger();
    pdl_wait();
    const int bh = blockIdx.x;
    const int b = bh / heads, h = bh % heads;
    const int d = threadIdx.x;
    const float* pp = part + (int64_t)bh * splits * (kDecHd + 2);
    float M = -INFINITY;
    for (int s = 0; s < splits; ++s) M = fmaxf(M, pp[s * (kDecHd + 2) + kDecHd]);
    float L = 0.0f, A = 0.0f;
    for (int s = 0; s < splits; ++s) {
        const float ms = pp[s * (kDecHd + 2) + kDecHd];
        const float c = (ms == -INFINITY) ? 0.0f : exp2f(ms - M);
        L += pp[s * (kDecHd + 2) + kDecHd + 1] * c;
        A += pp[s * (kDecHd + 2) + d] * c;
    }
    out[(int64_t)b * ldo + (int64_t)h * kDecHd + d] = __float2half_rn(L > 0.0f ? A / L : 0.0f);
}

__global__ void kv_append_kernel(const __half* __restrict__ kn, int64_t ldk, const __half* __restrict__ vn,
                                 int64_t ldv, __half* kc, __half* vc, int64_t cap, const int32_t* __restrict__ pos,
                                 int pos0, int kvh, int hd) {
    const int b = blockIdx.x;
    const int p = pos ? pos[b] : pos0;
    for (int i = threadIdx.x; i < kvh * hd; i += blockDim.x) {
        const int h = i / hd, d = i % hd;
        const int64_t dst = (((int64_t)b * kvh + h) * cap + p) * hd + d;
        kc[dst] = kn[(int64_t)b * ldk + i];
        vc[dst] = vn[(int64_t)b * ldv + i];
    }
}

static int64_t pad8(int64_t x) { return (x + 7) / 8 * 8; }

static int decode_splits(int bh, int ctx) {
    const int sms = num_sms();
    int s = 1;
    while (bh * s < sms * 6 && ctx / (s * 2) >= 256 && s < 32) s *= 2;
    return s;
}

}  // namespace npub

using namespace npub;

static size_t attn_s_bytes(int batch, int tokens, int heads) {
    const int64_t tp = pad8(tokens);
    return ((size_t)batch * heads * tokens * tp * 2 + 255) / 256 * 256;
}

extern "C" size_t npub_attention_workspace(int batch, int tokens, int heads, int head_dim) {
    if (batch <= 0 || tokens <= 0 || heads <= 0 || head_dim <= 0) return 0;
    if (head_dim == 128) return 0;  // fused flash-attention kernel (fmha.cu): no scratch
    const int64_t tp = pad8(tokens);
    // S/P [batch*heads, tokens, tp] + Vt [batch*heads, head_dim, tp] (kv_heads <= heads)
    const size_t v_bytes = ((size_t)batch * heads * head_dim * tp * 2 + 255) / 256 * 256;
    return attn_s_bytes(batch, tokens, heads) + v_bytes;
}

extern "C" int npub_attention_prefill(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                                      int64_t ldv, void* out, int64_t ldo, int batch, int tokens, int heads,
                                      int kv_heads, int head_dim, float scale, int causal, void* workspace,
                                      size_t workspace_bytes, void* stream) {
    NPUB_CHECK_ARG(batch >= 0 && tokens >= 0 && heads > 0 && kv_heads > 0 && heads % kv_heads == 0);
    if (tokens == 0 || batch == 0) return NPUB_OK;
    NPUB_CHECK_ARG(q && k && v && out);
    NPUB_CHECK_ARG(head_dim % 16 == 0 && head_dim > 0 && head_dim <= 256);
    NPUB_CHECK_ARG(ldq % 8 == 0 && ldk % 8 == 0 && ldv % 8 == 0);
    NPUB_CHECK_ARG(ldq >= (int64_t)heads * head_dim && ldk >= (int64_t)kv_heads * head_dim &&
                   ldv >= (int64_t)kv_heads * head_dim && ldo >= (int64_t)heads * head_dim);
    NPUB_CHECK_ARG(npub_aligned(q, 16) && npub_aligned(k, 16) && npub_aligned(v, 16));
    NPUB_CHECK_ARG((int64_t)batch * heads <= 65535 && (int64_t)batch * tokens <= 0x7fffffffLL);
    cudaStream_t st0 = reinterpret_cast<cudaStream_t>(stream);
    if (head_dim == 128)
        return fmha_prefill(q, ldq, k, ldk, v, ldv, out, ldo, batch, tokens, heads, kv_heads, scale, causal, st0);
    const size_t need = npub_attention_workspace(batch, tokens, heads, head_dim);
    if (!workspace || workspace_bytes < need) return NPUB_ERR_WORKSPACE;
    NPUB_CHECK_ARG(npub_aligned(workspace, 256));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int64_t tp = pad8(tokens);
    __half* S = reinterpret_cast<__half*>(workspace);
    __half* Vt = reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(workspace) + attn_s_bytes(batch, tokens, heads));
    const int group = heads / kv_heads;
    const int off = causal ? 0 : NPUB_NO_CAUSAL;
    const int rows_all = batch * tokens;

    // 1) S[b*H + h] = Q_{b,h} K_{b,h/group}^T, fp16, row stride tp.  z = b*H + h.
    {
        GemmParams p;
        memset(&p, 0, sizeof(p));
        int rc = make_tmap_3d(&p.tmA, false, q, (uint64_t)head_dim, (uint64_t)heads, (uint64_t)rows_all,
                              (uint64_t)head_dim, (uint64_t)ldq, 1, 128, true);
        if (rc) return rc;
        const int bt = pick_bt(tokens);
        rc = make_tmap_3d(&p.tmB, false, k, (uint64_t)head_dim, (uint64_t)kv_heads, (uint64_t)rows_all,
                          (uint64_t)head_dim, (uint64_t)ldk, 1, (uint32_t)bt, true);
        if (rc) return rc;
        p.a_rows = tokens;
        p.b_rows = tokens;
        p.k_tiles = (head_dim + 63) / 64;
        p.a_row_dim = 2;
        p.b_row_dim = 2;
        p.zmod = heads;
        p.za = ZMap{1, 0, tokens, 0};
        p.zb = ZMap{group, 0, tokens, 0};
        p.splits = 1;
        p.k_tiles_per_split = p.k_tiles;
        p.causal_mode = causal ? 1 : 0;
        p.causal_off = 0;
        p.out = S;
        p.o_sa = tp;
        p.o_sb = 1;
        p.o_zl = (int64_t)tokens * tp;
        p.o_zh = (int64_t)heads * tokens * tp;
        p.alpha = 1.0f;
        rc = run_gemm(p, false, bt, (tokens + 127) / 128, (tokens + bt - 1) / bt, batch * heads, st);
        if (rc) return rc;
    }
    // 2) P = softmax(S * scale) in place
    {
        int rc = npub_softmax_rows(S, S, tp, (int64_t)tokens * tp, batch * heads, tokens, tokens, scale, off, 0,
                                   stream);
        if (rc) return rc;
    }
    // 3) Vt[b*KVH + kvh] = V_{b,kvh}^T
    {
        dim3 grid((unsigned)((tp + 63) / 64), (unsigned)((head_dim + 63) / 64), (unsigned)(batch * kv_heads));
        transpose_heads_kernel<<<grid, dim3(32, 8), 0, st>>>(reinterpret_cast<const __half*>(v), ldv, tokens,
                                                             kv_heads, head_dim, Vt, tp);
        int rc = npub_internal_launch_status();
        if (rc) return rc;
    }
    // 4) O[b*T + t, h*hd + d] = P_{b,h} Vt_{b,h/group}^T
    {
        GemmParams p;
        memset(&p, 0, sizeof(p));
        int rc = make_tmap_3d(&p.tmA, false, S, (uint64_t)tokens, (uint64_t)tokens, (uint64_t)batch * heads,
                              (uint64_t)tp, (uint64_t)tokens * tp, 128, 1, true);
        if (rc) return rc;
        const int bt = pick_bt(head_dim);
        rc = make_tmap_3d(&p.tmB, false, Vt, (uint64_t)tokens, (uint64_t)head_dim, (uint64_t)batch * kv_heads,
                          (uint64_t)tp, (uint64_t)head_dim * tp, (uint32_t)bt, 1, true);
        if (rc) return rc;
        p.a_rows = tokens;
        p.b_rows = head_dim;
        p.k_tiles = (tokens + 63) / 64;
        p.a_row_dim = 1;
        p.b_row_dim = 1;
        p.zmod = heads;
        p.za = ZMap{1, heads, 0, 0};
        p.zb = ZMap{group, kv_heads, 0, 0};
        p.splits = 1;
        p.k_tiles_per_split = p.k_tiles;
        p.causal_mode = causal ? 2 : 0;
        p.causal_off = 0;
        p.out = out;
        p.o_sa = ldo;
        p.o_sb = 1;
        p.o_zl = head_dim;
        p.o_zh = (int64_t)tokens * ldo;
        p.alpha = 1.0f;
        rc = run_gemm(p, false, bt, (tokens + 127) / 128, (head_dim + bt - 1) / bt, batch * heads, st);
        if (rc) return rc;
    }
    return NPUB_OK;
}

extern "C" size_t npub_attention_decode_workspace(int batch, int heads, int ctx_len, int head_dim) {
    if (batch <= 0 || heads <= 0 || head_dim != kDecHd) return 0;
    // the persistent kernel's published pieces (group <= 8) or the split kernel's partials
    const size_t ps = (size_t)ps_max_ctas() * (heads < 8 ? heads : 8) * (kDecHd + 2) * sizeof(float);
    const int s = ctx_len > 0 ? decode_splits(batch * heads, ctx_len) : 1;
    const size_t split = s > 1 ? (size_t)batch * heads * s * (kDecHd + 2) * sizeof(float) : 0;
    return ps > split ? ps : split;
}

extern "C" int npub_attention_decode(const void* q, int64_t ldq, const void* k_cache, const void* v_cache, int64_t cap,
                                     const int32_t* lens, int ctx_len, void* out, int64_t ldo, int batch, int heads,
                                     int kv_heads, int head_dim, float scale, void* workspace, size_t workspace_bytes,
                                     void* stream) {
    NPUB_CHECK_ARG(batch >= 0 && heads > 0 && kv_heads > 0 && heads % kv_heads == 0);
    if (batch == 0) return NPUB_OK;
    if (head_dim != kDecHd) return NPUB_ERR_UNSUPPORTED;
    NPUB_CHECK_ARG(q && k_cache && v_cache && out && ctx_len >= 0 && cap >= ctx_len);
    NPUB_CHECK_ARG(ldq % 8 == 0 && ldq >= (int64_t)heads * head_dim && ldo >= (int64_t)heads * head_dim);
    NPUB_CHECK_ARG(npub_aligned(q, 16) && npub_aligned(k_cache, 16) && npub_aligned(v_cache, 16));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int bh = batch * heads;
    const int ctx_max = ctx_len > 0 ? ctx_len : 1;
    const int splits = decode_splits(bh, ctx_max);
    DecodeArgs a;
    a.q = reinterpret_cast<const __half*>(q);
    a.ldq = ldq;
    a.kc = reinterpret_cast<const __half*>(k_cache);
    a.vc = reinterpret_cast<const __half*>(v_cache);
    a.cap = cap;
    a.lens = lens;
    a.ctx = ctx_len;
    a.out = reinterpret_cast<__half*>(out);
    a.ldo = ldo;
    a.heads = heads;
    a.kv_heads = kv_heads;
    a.splits = splits;
    a.chunk = (ctx_max + splits - 1) / splits;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.part = nullptr;
    a.batch = batch;
    a.err = npub_internal_device_error_word();
    a.wait_ns = npub_internal_wait_limit_ns();
    a.tail_first = 0;
    a.tail_parts = 1;
    a.kv_evict_first = npub_internal_l2_evict_first() ? 1 : 0;
    const int group = heads / kv_heads;
    const int64_t items = (int64_t)batch * kv_heads;
    const bool streaming = group >= 1 && group <= 8;
    // Ring depth (kernel A/B on one B200, L2 flushed): two 32 KB stages beat
    // three for grouped heads (64 seq x 8 kv heads x 4096 keys 363 -> 343 us,
    // 16 x 8 x 4096 112 -> 103 us) and for short contexts (128 x 32 x 512 keys
    // 166 -> 160 us; the batch-32 x 1088-key layer step -0.9 %), three for one
    // head per group at long contexts (64 x 32 x 4096 keys 596 vs 606 us).
    const int ns = (group > 1 || ctx_max <= 2048) ? 2 : 3;
    // Schedules, by the number of (sequence, kv head) items (measured on B200):
    //  * >= 6 per SM: one streaming CTA per item;
    //  * 32 .. 6 per SM: the persistent grid over the stage list (4-24 % faster
    //    than context splits and a combine pass there);
    //  * fewer: one streaming CTA per (item, context split) and a combine pass
    //    (a persistent finisher would merge ~40 pieces one after another).
    if (streaming && items < 6LL * num_sms() && items >= 32 && batch <= kPsMaxSeq &&
        items * ((cap + kStKeys - 1) / kStKeys) < 0x7fffffffLL) {
        a.part = reinterpret_cast<float*>(workspace);
        const int64_t stages = items * (((ctx_len > 0 ? (int64_t)ctx_len : cap) + kStKeys - 1) / kStKeys);
        return ns == 2 ? persist_by_group<2>(group, a, stages, workspace_bytes, st)
                       : persist_by_group<3>(group, a, stages, workspace_bytes, st);
    }
    if (splits > 1) {
        const size_t need = (size_t)bh * splits * (kDecHd + 2) * sizeof(float);
        if (!workspace || workspace_bytes < need) return NPUB_ERR_WORKSPACE;
        a.part = reinterpret_cast<float*>(workspace);
    }
    int rc;
    if (streaming) {
        rc = ns == 2 ? stream_by_group<2>(group, a, batch, kv_heads, splits, workspace, workspace_bytes, st)
                     : stream_by_group<3>(group, a, batch, kv_heads, splits, workspace, workspace_bytes, st);
    } else {
        decode_attn_kernel<<<dim3(bh, splits), kDecWarps * 32, 0, st>>>(a);
        rc = npub_internal_launch_status();
    }
    if (rc || splits == 1) return rc;
    return launch_pdl(decode_combine_kernel, dim3(bh), dim3(kDecHd), 0, st, (const float*)a.part, splits, heads,
                      a.out, ldo);
}

// Clears the persistent decode kernel's piece flags (a finisher whose wait
// gave up leaves them set).
int npub_internal_decode_flags_reset() {
    const uint32_t zero[kPsMaxCtas] = {};
    cudaError_t e = cudaMemcpyToSymbol(g_decode_piece_flag, zero, sizeof(zero));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_decode_tail_cnt, zero, sizeof(zero));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        npub_internal_set_cuda_error(e);
        return NPUB_ERR_CUDA;
    }
    return NPUB_OK;
}

extern "C" int npub_kv_append(const void* k_new, int64_t ldk, const void* v_new, int64_t ldv, void* k_cache,
                              void* v_cache, int64_t cap, const int32_t* pos, int pos0, int batch, int kv_heads,
                              int head_dim, void* stream) {
    NPUB_CHECK_ARG(batch >= 0 && kv_heads > 0 && head_dim > 0);
    if (batch == 0) return NPUB_OK;
    NPUB_CHECK_ARG(k_new && v_new && k_cache && v_cache);
    NPUB_CHECK_ARG(pos || (pos0 >= 0 && pos0 < cap));
    NPUB_CHECK_ARG(ldk >= (int64_t)kv_heads * head_dim && ldv >= (int64_t)kv_heads * head_dim);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    kv_append_kernel<<<batch, 256, 0, st>>>(reinterpret_cast<const __half*>(k_new), ldk,
                                            reinterpret_cast<const __half*>(v_new), ldv,
                                            reinterpret_cast<__half*>(k_cache), reinterpret_cast<__half*>(v_cache), cap,
                                            pos, pos0, kv_heads, head_dim);
    return npub_internal_launch_status();
}

// Bandwidth-bound Llama-layer vector kernels for sm_100a: RMSNorm (with the
// fused residual add), SwiGLU, causal row softmax, RoPE, and the W8
// quantiser.  All use 128-bit coalesced loads/stores of fp16 and fp32 math
// with warp-shuffle reductions.
#include "common.cuh"

#include <cmath>

#include <math.h>

namespace npub {

constexpr int kVec = 8;  // fp16 elements per 128-bit access

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 t = __half22float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    return u;
}

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int i = 0; i < NT / 32; ++i) t += red[i];
    return t;
}

template <int NT>
__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = red[0];
#pragma unroll
    for (int i = 1; i < NT / 32; ++i) t = fmaxf(t, red[i]);
    return t;
}

// ------------------------------------------------------------ RMSNorm
// One CTA per row; up to CH chunks of 8 elements per thread kept in registers.
template <int NT, int CH>
__global__ void __launch_bounds__(NT) rmsnorm_kernel(const __half* __restrict__ x, int64_t ldx,
                                                     const __half* __restrict__ r, int64_t ldr, __half* xo,
                                                     int64_t ldxo, const __half* __restrict__ gamma,
                                                     __half* __restrict__ y, int64_t ldy, int d, float eps) {
    pdl_trigger();
    pdl_wait();
    __shared__ float red[NT / 32];
    const int row = blockIdx.x;
    const int nch = d / kVec;
    const __half* xr = x + (int64_t)row * ldx;
    float v[CH][8];
    float ss = 0.0f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const int ch = threadIdx.x + c * NT;
        if (ch < nch) {
            uint4 u = *reinterpret_cast<const uint4*>(xr + ch * kVec);
            unpack8(u, v[c]);
            if (r) {
                float rv[8];
                unpack8(*reinterpret_cast<const uint4*>(r + (int64_t)row * ldr + ch * kVec), rv);
#pragma unroll
                for (int i = 0; i < 8; ++i) v[c][i] = __half2float(__float2half_rn(v[c][i] + rv[i]));
                *reinterpret_cast<uint4*>(xo + (int64_t)row * ldxo + ch * kVec) = pack8(v[c]);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) ss += v[c][i] * v[c][i];
        }
    }
    const float tot = block_sum<NT>(ss, red);
    const float inv = 1.0f / sqrtf(tot / (float)d + eps);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const int ch = threadIdx.x + c * NT;
        if (ch < nch) {
            float g[8], o[8];
            unpack8(*reinterpret_cast<const uint4*>(gamma + ch * kVec), g);
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = (v[c][i] * inv) * g[i];
            *reinterpret_cast<uint4*>(y + (int64_t)row * ldy + ch * kVec) = pack8(o);
        }
    }
}

// One warp per row, two rows per CTA, for rows of up to 32 x 8 x CPL elements
// (d = 4096: 16 16-byte chunks per lane).  Every load of the row is issued
// before the first is used, the sum of squares is a warp-shuffle reduction
// (no block barrier), and the row stays in registers as packed fp16 between
// the two passes.  At 2048 x 4096 it measured 10.6 us (one CTA per row with
// block reductions: 11.1 us; persistent double-buffered CTAs: 10.0-19.6 us).
// HAS_R: the residual-add form (x and r of the row in registers at once);
// without it the kernel fits ten 64-thread CTAs per SM, so a 2048-row
// prompt is one wave of 2048 warps with every load of its rows in flight.
template <int CPL, bool HAS_R>
__global__ void __launch_bounds__(64, HAS_R ? 1 : 10) rmsnorm_warp_kernel(const __half* __restrict__ x, int64_t ldx,
                                                         const __half* __restrict__ r, int64_t ldr, __half* xo,
                                                         int64_t ldxo, const __half* __restrict__ gamma,
                                                         __half* __restrict__ y, int64_t ldy, int rows, int d,
                                                         float eps) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 2 + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int nch = d / kVec;
    const __half* xr = x + (int64_t)row * ldx;
    uint4 v[CPL];
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
        const int ch = lane + 32 * j;
        if (ch < nch) v[j] = *reinterpret_cast<const uint4*>(xr + ch * kVec);
    }
    if (HAS_R) {
        const __half* rr = r + (int64_t)row * ldr;
        uint4 w[CPL];
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
            const int ch = lane + 32 * j;
            if (ch < nch) w[j] = *reinterpret_cast<const uint4*>(rr + ch * kVec);
        }
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
            const int ch = lane + 32 * j;
            if (ch < nch) {
                float a[8], b[8];
                unpack8(v[j], a);
                unpack8(w[j], b);
#pragma unroll
                for (int i = 0; i < 8; ++i) a[i] = a[i] + b[i];
                v[j] = pack8(a);  // fp16(x + r), the residual stream
                *reinterpret_cast<uint4*>(xo + (int64_t)row * ldxo + ch * kVec) = v[j];
            }
        }
    }
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
        if (lane + 32 * j < nch) {
            float a[8];
            unpack8(v[j], a);
#pragma unroll
            for (int i = 0; i < 8; ++i) ss += a[i] * a[i];
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.0f / sqrtf(ss / (float)d + eps);
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
        const int ch = lane + 32 * j;
        if (ch < nch) {
            float a[8], g[8], o[8];
            unpack8(v[j], a);
            unpack8(__ldg(reinterpret_cast<const uint4*>(gamma + ch * kVec)), g);
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = (a[i] * inv) * g[i];
            *reinterpret_cast<uint4*>(y + (int64_t)row * ldy + ch * kVec) = pack8(o);
        }
    }
}

// ------------------------------------------------------------ SwiGLU
__global__ void swiglu_vec_kernel(const __half* __restrict__ g, int64_t ldg, const __half* __restrict__ u,
                                  int64_t ldu, __half* __restrict__ h, int64_t ldh, int rows, int cols) {
    pdl_trigger();
    pdl_wait();
    const int cpr = cols / kVec;
    const int64_t total = (int64_t)rows * cpr;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int rr = (int)(i / cpr), c = (int)(i - (int64_t)rr * cpr) * kVec;
        float gv[8], uv[8], o[8];
        unpack8(*reinterpret_cast<const uint4*>(g + (int64_t)rr * ldg + c), gv);
        unpack8(*reinterpret_cast<const uint4*>(u + (int64_t)rr * ldu + c), uv);
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = swiglu_f(gv[k], uv[k]);
        *reinterpret_cast<uint4*>(h + (int64_t)rr * ldh + c) = pack8(o);
    }
}

__global__ void swiglu_scalar_kernel(const __half* __restrict__ g, int64_t ldg, const __half* __restrict__ u,
                                     int64_t ldu, __half* __restrict__ h, int64_t ldh, int rows, int cols) {
    const int64_t total = (int64_t)rows * cols;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int rr = (int)(i / cols), c = (int)(i - (int64_t)rr * cols);
        const float gv = __half2float(g[(int64_t)rr * ldg + c]), uv = __half2float(u[(int64_t)rr * ldu + c]);
        h[(int64_t)rr * ldh + c] = __float2half_rn(swiglu_f(gv, uv));
    }
}

// ------------------------------------------------------------ residual add
__global__ void add_vec_kernel(const __half* __restrict__ a, int64_t lda, const __half* __restrict__ b, int64_t ldb,
                               __half* __restrict__ o, int64_t ldo, int rows, int cols) {
    pdl_trigger();
    pdl_wait();
    const int cpr = cols / kVec;
    const int64_t total = (int64_t)rows * cpr;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int rr = (int)(i / cpr), c = (int)(i - (int64_t)rr * cpr) * kVec;
        float av[8], bv[8], ov[8];
        unpack8(*reinterpret_cast<const uint4*>(a + (int64_t)rr * lda + c), av);
        unpack8(*reinterpret_cast<const uint4*>(b + (int64_t)rr * ldb + c), bv);
#pragma unroll
        for (int k = 0; k < 8; ++k) ov[k] = av[k] + bv[k];
        *reinterpret_cast<uint4*>(o + (int64_t)rr * ldo + c) = pack8(ov);
    }
}

__global__ void add_scalar_kernel(const __half* __restrict__ a, int64_t lda, const __half* __restrict__ b, int64_t ldb,
                                  __half* __restrict__ o, int64_t ldo, int rows, int cols) {
    const int64_t total = (int64_t)rows * cols;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int rr = (int)(i / cols), c = (int)(i - (int64_t)rr * cols);
        o[(int64_t)rr * ldo + c] =
            __float2half_rn(__half2float(a[(int64_t)rr * lda + c]) + __half2float(b[(int64_t)rr * ldb + c]));
    }
}

// ------------------------------------------------------------ softmax
// One CTA per row.  Valid columns: [0, min(cols, r + off + 1)) when causal.
// Masked columns are written as zero up to zend.
template <int NT, int CH>
__global__ void __launch_bounds__(NT) softmax_kernel(const __half* s, __half* p, int64_t ld, int64_t bstride,
                                                     int rows, int cols, float scale, int off, int zero_full) {
    __shared__ float red[NT / 32];
    const int rr = blockIdx.x % rows;
    const int b = blockIdx.x / rows;
    const __half* sr = s + (int64_t)b * bstride + (int64_t)rr * ld;
    __half* pr = p + (int64_t)b * bstride + (int64_t)rr * ld;
    int valid = cols, zend = cols;
    if (off >= 0) {
        valid = min(cols, rr + off + 1);
        if (!zero_full) {
            const int a0 = (rr / 128) * 128;
            zend = min(cols, ((a0 + 128 + off + 63) / 64) * 64);
        }
    }
    const float l2e = 1.4426950408889634f;
    const float sc = scale * l2e;  // work in base 2: exp(x) = exp2(x * log2 e)
    float v[CH][8];
    float mx = -INFINITY;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const int e0 = (threadIdx.x + c * NT) * kVec;
        if (e0 < valid) {
            unpack8(*reinterpret_cast<const uint4*>(sr + e0), v[c]);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                v[c][i] = (e0 + i < valid) ? v[c][i] * sc : -INFINITY;
                mx = fmaxf(mx, v[c][i]);
            }
        }
    }
    mx = block_max<NT>(mx, red);
    float sum = 0.0f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const int e0 = (threadIdx.x + c * NT) * kVec;
        if (e0 < valid) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                v[c][i] = (e0 + i < valid) ? exp2f(v[c][i] - mx) : 0.0f;
                sum += v[c][i];
            }
        }
    }
    sum = block_sum<NT>(sum, red);
    const float inv = 1.0f / sum;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const int e0 = (threadIdx.x + c * NT) * kVec;
        if (e0 < zend) {
            float o[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = (e0 < valid) ? v[c][i] * inv : 0.0f;
            if (e0 + 8 <= zend) {
                *reinterpret_cast<uint4*>(pr + e0) = pack8(o);
            } else {
                for (int i = 0; i < 8 && e0 + i < zend; ++i) pr[e0 + i] = __float2half_rn(o[i]);
            }
        }
    }
}

// One warp per row for rows of up to 32 x 8 x CPL columns (2048: 8 16-byte
// chunks per lane).  Only the unmasked chunks are read (streaming loads); the
// row is kept packed in registers through the max, sum and scale passes, the
// exponentials are recomputed in the last pass with the hardware ex2
// (MUFU.EX2, ~2 ulp of fp32, far below the fp16 output; the fused attention
// kernel uses the same instruction) rather than held as fp32, and the masked
// part up to `zend` is written as zeros with streaming stores.  Measured at
// 32 x 2048 x 2048 causal: 74.6 us (0.83 of the copy bandwidth for the 403 MB
// moved) against 95 us with exp2f and 134 us for softmax_kernel.
template <int CPL>
__global__ void __launch_bounds__(256) softmax_warp_kernel(const __half* s, __half* p, int64_t ld, int64_t bstride,
                                                         int rows, int nrows_total, int cols, float scale, int off,
                                                         int zero_full) {
    const int lane = threadIdx.x & 31;
    const int gr = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (gr >= nrows_total) return;
    const int rr = gr % rows, b = gr / rows;
    const __half* sr = s + (int64_t)b * bstride + (int64_t)rr * ld;
    __half* pr = p + (int64_t)b * bstride + (int64_t)rr * ld;
    int valid = cols, zend = cols;
    if (off >= 0) {
        valid = min(cols, rr + off + 1);
        if (!zero_full) {
            const int a0 = (rr / 128) * 128;
            zend = min(cols, ((a0 + 128 + off + 63) / 64) * 64);
        }
    }
    const float sc = scale * 1.4426950408889634f;  // exp(x) = exp2(x log2 e)
    uint4 v[CPL];
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
        const int e0 = (lane + 32 * j) * kVec;
        if (e0 < valid) v[j] = __ldcs(reinterpret_cast<const uint4*>(sr + e0));
    }
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
        const int e0 = (lane + 32 * j) * kVec;
        if (e0 < valid) {
            float a[8];
            unpack8(v[j], a);
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (e0 + i < valid) mx = fmaxf(mx, a[i] * sc);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
        const int e0 = (lane + 32 * j) * kVec;
        if (e0 < valid) {
            float a[8];
            unpack8(v[j], a);
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (e0 + i < valid) sum += ex2_approx(a[i] * sc - mx);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = 1.0f / sum;
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
        const int e0 = (lane + 32 * j) * kVec;
        if (e0 < zend) {
            float o[8];
            if (e0 < valid) {
                float a[8];
                unpack8(v[j], a);
#pragma unroll
                for (int i = 0; i < 8; ++i) o[i] = (e0 + i < valid) ? ex2_approx(a[i] * sc - mx) * inv : 0.0f;
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) o[i] = 0.0f;
            }
            if (e0 + 8 <= zend) {
                __stcs(reinterpret_cast<uint4*>(pr + e0), pack8(o));
            } else {
                for (int i = 0; i < 8 && e0 + i < zend; ++i) pr[e0 + i] = __float2half_rn(o[i]);
            }
        }
    }
}

// ------------------------------------------------------------ RoPE
// Frequency i of a head: theta^(-2i/hd), or inv_freq[i] when a table is given
// (Llama-3 scaled frequencies, legalize.py:50-64).
__device__ __forceinline__ float rope_freq(int k, int hd, float log2_theta, const float* __restrict__ inv_freq) {
    return inv_freq ? __ldg(inv_freq + k) : exp2f(-(2.0f * (float)k / (float)hd) * log2_theta);
}

__global__ void rope_kernel(__half* x, int64_t ldx, int tokens, int heads, int hd, const int32_t* __restrict__ pos,
                            int pos0, float log2_theta, const float* __restrict__ inv_freq) {
    const int half = hd / 2;
    const int64_t total = (int64_t)tokens * heads * half;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int k = (int)(i % half);
        const int64_t th = i / half;
        const int h = (int)(th % heads), t = (int)(th / heads);
        const int p = pos ? pos[t] : pos0 + t;
        float sn, cs;
        sincosf((float)p * rope_freq(k, hd, log2_theta, inv_freq), &sn, &cs);
        __half* row = x + (int64_t)t * ldx + (int64_t)h * hd;
        const float x1 = __half2float(row[k]), x2 = __half2float(row[k + half]);
        row[k] = __float2half_rn(x1 * cs - x2 * sn);
        row[k + half] = __float2half_rn(x2 * cs + x1 * sn);
    }
}

// Vectorised RoPE: one CTA per token; the token's cos/sin for the hd/2
// frequencies are computed once into shared memory, then every head's pairs
// (x[i], x[i + hd/2]) are rotated 8 at a time with 128-bit accesses.
__global__ void rope_vec_kernel(__half* x, int64_t ldx, int heads, int hd, const int32_t* __restrict__ pos, int pos0,
                                float log2_theta, const float* __restrict__ inv_freq) {
    pdl_trigger();
    pdl_wait();
    __shared__ float cs[256], sn[256];
    const int t = blockIdx.x;
    const int half = hd / 2;
    const int p = pos ? pos[t] : pos0 + t;
    for (int k = threadIdx.x; k < half; k += blockDim.x) {
        float sv, cv;
        sincosf((float)p * rope_freq(k, hd, log2_theta, inv_freq), &sv, &cv);
        cs[k] = cv;
        sn[k] = sv;
    }
    __syncthreads();
    __half* row = x + (int64_t)t * ldx;
    const int per_head = half / 8;
    for (int i = threadIdx.x; i < heads * per_head; i += blockDim.x) {
        const int hh = i / per_head, k0 = (i - hh * per_head) * 8;
        __half* a = row + (int64_t)hh * hd + k0;
        float x1[8], x2[8], y1[8], y2[8];
        unpack8(*reinterpret_cast<const uint4*>(a), x1);
        unpack8(*reinterpret_cast<const uint4*>(a + half), x2);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float c = cs[k0 + e], sv = sn[k0 + e];
            y1[e] = x1[e] * c - x2[e] * sv;
            y2[e] = x2[e] * c + x1[e] * sv;
        }
        *reinterpret_cast<uint4*>(a) = pack8(y1);
        *reinterpret_cast<uint4*>(a + half) = pack8(y2);
    }
}

// Decode-step RoPE fused with the KV-cache append: CTA (t, g) takes heads
// [8 g, 8 g + 8) of token t's fused QKV row (q heads | k heads | v heads).
// q and k heads are rotated in place exactly as rope_vec_kernel does; k and v
// heads are also written to cache[t, h, pos[t], :]; CTA (t, 0) writes
// lens[t] = pos[t] + 1 (the attention length of the step).
// Row t belongs to sequence t / tps (tps = 1 for a decode step); blockIdx.y
// takes heads [hpb * y, hpb * y + hpb).  A position outside [0, cap) is
// rotated but not stored.
__global__ void rope_kv_append_kernel(__half* x, int64_t ldx, int hq, int hk, int hd, int tps, int hpb,
                                      const int32_t* __restrict__ pos, float log2_theta,
                                      const float* __restrict__ inv_freq, __half* __restrict__ kc,
                                      __half* __restrict__ vc, int64_t cap, int32_t* __restrict__ lens) {
    pdl_trigger();
    pdl_wait();
    __shared__ float cs[256], sn[256];
    const int t = blockIdx.x;
    const int half = hd / 2;
    const int p = pos[t];
    if (lens && blockIdx.y == 0 && threadIdx.x == 0) lens[t] = p + 1;
    for (int k = threadIdx.x; k < half; k += blockDim.x) {
        float sv, cv;
        sincosf((float)p * rope_freq(k, hd, log2_theta, inv_freq), &sv, &cv);
        cs[k] = cv;
        sn[k] = sv;
    }
    __syncthreads();
    __half* row = x + (int64_t)t * ldx;
    const int64_t seq = t / tps;
    const bool store = p >= 0 && (int64_t)p < cap;
    const int h0 = blockIdx.y * hpb;
    const int h1 = min(h0 + hpb, hq + 2 * hk);
    const int per_head = half / 8;
    for (int i = threadIdx.x; i < (h1 - h0) * per_head; i += blockDim.x) {
        const int hh = h0 + i / per_head, k0 = (i % per_head) * 8;
        __half* a = row + (int64_t)hh * hd + k0;
        const uint4 r1 = *reinterpret_cast<const uint4*>(a);
        const uint4 r2 = *reinterpret_cast<const uint4*>(a + half);
        uint4 o1 = r1, o2 = r2;
        if (hh < hq + hk) {  // q and k heads are rotated
            float x1[8], x2[8], y1[8], y2[8];
            unpack8(r1, x1);
            unpack8(r2, x2);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float c = cs[k0 + e], sv = sn[k0 + e];
                y1[e] = x1[e] * c - x2[e] * sv;
                y2[e] = x2[e] * c + x1[e] * sv;
            }
            o1 = pack8(y1);
            o2 = pack8(y2);
            *reinterpret_cast<uint4*>(a) = o1;
            *reinterpret_cast<uint4*>(a + half) = o2;
        }
        if (hh >= hq && store) {  // k and v heads go to the caches
            const bool isk = hh < hq + hk;
            const int kvh = isk ? hh - hq : hh - hq - hk;
            __half* dst = (isk ? kc : vc) + ((seq * hk + kvh) * cap + p) * hd + k0;
            *reinterpret_cast<uint4*>(dst) = o1;
            *reinterpret_cast<uint4*>(dst + half) = o2;
        }
    }
}

// ------------------------------------------------------------ embedding / argmax
// out[r, :] = table[ids[r], :]; ids outside [0, vocab) give a zero row.
__global__ void embed_kernel(const int32_t* __restrict__ ids, const __half* __restrict__ table, int64_t ldt,
                             int vocab, int d, __half* __restrict__ out, int64_t ldo) {
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x;
    const int id = ids[r];
    const bool ok = id >= 0 && id < vocab;
    const uint4* src = reinterpret_cast<const uint4*>(table + (int64_t)(ok ? id : 0) * ldt);
    uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)r * ldo);
    for (int c = threadIdx.x; c < d / kVec; c += blockDim.x) dst[c] = ok ? src[c] : make_uint4(0, 0, 0, 0);
}

// Row argmax over fp16 logits: the largest value and its smallest index.
// Order-preserving 64-bit key of (value, index): the float's bits made
// unsigned-monotone in the high word, 0xffffffff - index in the low word, so
// the largest key is the largest value with the smallest index.
__device__ __forceinline__ uint64_t argmax_key(float v, int32_t i) {
    const uint32_t u = __float_as_uint(v);
    const uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((uint64_t)o << 32) | (uint64_t)(0xffffffffu - (uint32_t)i);
}

__global__ void argmax_kernel(const __half* __restrict__ x, int64_t ldx, int cols, int32_t* __restrict__ idx,
                              float* __restrict__ val, uint64_t* __restrict__ key, int32_t key_off) {
    pdl_trigger();
    pdl_wait();
    __shared__ float sv[32];
    __shared__ int si[32];
    const __half* row = x + (int64_t)blockIdx.x * ldx;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    auto take = [&](float v, int c) {
        if (v > best || (v == best && c < bi)) {
            best = v;
            bi = c;
        }
    };
    int c0 = 0;
    if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) {
        // 16-byte loads, four in flight per thread (a row is a few hundred
        // vectors per warp: one pass of latency-bound rounds)
        const int nv = cols / 8;
        const uint4* rv = reinterpret_cast<const uint4*>(row);
        for (int v0 = threadIdx.x; v0 < nv; v0 += 4 * (int)blockDim.x) {
            uint4 u[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int v = v0 + k * (int)blockDim.x;
                u[k] = v < nv ? __ldg(rv + v) : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int v = v0 + k * (int)blockDim.x;
                if (v < nv) {
                    const __half2* h2 = reinterpret_cast<const __half2*>(&u[k]);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f = __half22float2(h2[e]);
                        take(f.x, 8 * v + 2 * e);
                        take(f.y, 8 * v + 2 * e + 1);
                    }
                }
            }
        }
        c0 = nv * 8;
    }
    for (int c = c0 + threadIdx.x; c < cols; c += blockDim.x) take(__half2float(row[c]), c);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) {
            best = ov;
            bi = oi;
        }
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) {
        sv[w] = best;
        si[w] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < (int)(blockDim.x >> 5); ++i)
            if (sv[i] > best || (sv[i] == best && si[i] < bi)) {
                best = sv[i];
                bi = si[i];
            }
        if (idx) idx[blockIdx.x] = bi;
        if (val) val[blockIdx.x] = best;
        if (key) key[blockIdx.x] = argmax_key(best, bi + key_off);
    }
}

// ids[b] = the index of the largest key[r * rows + b] over r < ranks.
__global__ void select_keys_kernel(const uint64_t* __restrict__ key, int ranks, int rows, int32_t* __restrict__ ids) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= rows) return;
    uint64_t best = key[b];
    for (int r = 1; r < ranks; ++r) {
        const uint64_t k = key[(int64_t)r * rows + b];
        best = k > best ? k : best;
    }
    ids[b] = (int32_t)(0xffffffffu - (uint32_t)(best & 0xffffffffu));
}

// ------------------------------------------------------------ quantiser
// W [K, N] fp32 -> Wq [N, K] int8 + s [N] fp16.  One CTA per 32 columns:
// pass 1 column absmax (coalesced over n), pass 2 writes K-major rows via smem.
__global__ void quantize_w8_kernel(const float* __restrict__ W, int64_t ldw, int K, int N, int8_t* __restrict__ q,
                                   int64_t ldq, __half* __restrict__ s) {
    __shared__ float colmax[8][32];
    __shared__ float sinv[32];
    __shared__ int8_t tile[32][64 + 4];
    const int n0 = blockIdx.x * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
    const int n = n0 + tx;
    float m = 0.0f;
    if (n < N)
        for (int k = ty; k < K; k += 8) m = fmaxf(m, fabsf(W[(int64_t)k * ldw + n]));
    colmax[ty][tx] = m;
    __syncthreads();
    if (ty == 0) {
        float mm = colmax[0][tx];
        for (int i = 1; i < 8; ++i) mm = fmaxf(mm, colmax[i][tx]);
        const __half sh = __float2half_rn(mm / 127.0f);
        const float sf = __half2float(sh);
        sinv[tx] = sf;
        if (n < N) s[n] = sh;
    }
    __syncthreads();
    for (int k0 = 0; k0 < K; k0 += 64) {
        // load 64 x 32 block, quantise, transpose through smem
        for (int kk = ty; kk < 64; kk += 8) {
            const int k = k0 + kk;
            int8_t qv = 0;
            if (n < N && k < K) {
                const float sf = sinv[tx];
                if (sf > 0.0f) {
                    float t = rintf(W[(int64_t)k * ldw + n] / sf);
                    t = fminf(127.0f, fmaxf(-127.0f, t));
                    qv = (int8_t)(int)t;
                }
            }
            tile[tx][kk] = qv;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < 32 * 64; i += 256) {
            const int nn = i / 64, kk = i % 64;
            if (n0 + nn < N && k0 + kk < K) q[(int64_t)(n0 + nn) * ldq + k0 + kk] = tile[nn][kk];
        }
        __syncthreads();
    }
}

static int grid_for(int64_t work, int threads) {
    int64_t b = (work + threads - 1) / threads;
    const int64_t cap = 148LL * 16;
    if (b > cap) b = cap;
    if (b < 1) b = 1;
    return (int)b;
}

// Inputs of an RMSNorm folded into the next W8A16 GEMM (npub_w8a16_gemm_rms):
// G = fp16(x * gamma) and, per 32 columns (chunk c), ss[c * ss_ld + row] =
// sum of x^2.  A lane holds 8 columns, four lanes a chunk.
__global__ void __launch_bounds__(256) rms_parts_kernel(const __half* __restrict__ x, int64_t ldx,
                                                        const __half* __restrict__ gamma, __half* __restrict__ G,
                                                        int64_t ldg, float* __restrict__ ss, int64_t ss_ld, int d) {
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int c0 = warp * 256; c0 < d; c0 += nw * 256) {
        const int col = c0 + lane * 8;
        float s = 0.0f;
        if (col < d) {
            float v[8], g[8], o[8];
            unpack8(*reinterpret_cast<const uint4*>(x + (int64_t)row * ldx + col), v);
            unpack8(*reinterpret_cast<const uint4*>(gamma + col), g);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                s += v[i] * v[i];
                o[i] = v[i] * g[i];
            }
            *reinterpret_cast<uint4*>(G + (int64_t)row * ldg + col) = pack8(o);
        }
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        if ((lane & 3) == 0 && col < d) ss[(int64_t)(col / 32) * ss_ld + row] = s;
    }
}

}  // namespace npub

using namespace npub;

extern "C" int npub_rmsnorm(const void* x, int64_t ldx, const void* residual, int64_t ldr, void* x_out, int64_t ldxo,
                            const void* gamma, void* y, int64_t ldy, int rows, int d, float eps, void* stream) {
    NPUB_CHECK_ARG(rows >= 0 && d > 0);
    if (rows == 0) return NPUB_OK;
    NPUB_CHECK_ARG(x && gamma && y);
    NPUB_CHECK_ARG(d % kVec == 0 && ldx % kVec == 0 && ldy % kVec == 0 && ldx >= d && ldy >= d);
    NPUB_CHECK_ARG(npub_aligned(x, 16) && npub_aligned(y, 16) && npub_aligned(gamma, 16));
    if (residual) {
        NPUB_CHECK_ARG(x_out && ldr % kVec == 0 && ldxo % kVec == 0 && ldr >= d && ldxo >= d);
        NPUB_CHECK_ARG(npub_aligned(residual, 16) && npub_aligned(x_out, 16));
    }
    NPUB_CHECK_ARG(d <= 8 * 256 * 8);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const __half* xh = reinterpret_cast<const __half*>(x);
    const __half* rh = reinterpret_cast<const __half*>(residual);
    __half* xoh = reinterpret_cast<__half*>(x_out);
    const __half* gh = reinterpret_cast<const __half*>(gamma);
    __half* yh = reinterpret_cast<__half*>(y);
    const int nch = d / kVec;
#define NPUB_RMSW(C)                                                                                              \
    (rh ? launch_pdl(rmsnorm_warp_kernel<C, true>, dim3((rows + 1) / 2), dim3(64), 0, st, xh, ldx, rh, ldr, xoh, \
                     ldxo, gh, yh, ldy, rows, d, eps)                                                           \
        : launch_pdl(rmsnorm_warp_kernel<C, false>, dim3((rows + 1) / 2), dim3(64), 0, st, xh, ldx, rh, ldr,   \
                     xoh, ldxo, gh, yh, ldy, rows, d, eps))
    if (nch <= 64) return NPUB_RMSW(2);
    if (nch <= 128) return NPUB_RMSW(4);
    if (nch <= 256) return NPUB_RMSW(8);
    if (nch <= 512) return NPUB_RMSW(16);
#undef NPUB_RMSW
#define NPUB_RMS(NT, V) launch_pdl(rmsnorm_kernel<NT, V>, dim3(rows), dim3(NT), 0, st, xh, ldx, rh, ldr, xoh, ldxo, gh, \
                                   yh, ldy, d, eps)
    if (nch <= 128) return NPUB_RMS(128, 1);
    if (nch <= 256) return NPUB_RMS(256, 1);
    if (nch <= 512) return NPUB_RMS(256, 2);
    if (nch <= 1024) return NPUB_RMS(256, 4);
    return NPUB_RMS(256, 8);
#undef NPUB_RMS
}

extern "C" int npub_rmsnorm_parts(const void* x, int64_t ldx, const void* gamma, void* G, int64_t ldg, float* ss,
                                  int64_t ss_ld, int rows, int d, void* stream) {
    NPUB_CHECK_ARG(rows >= 0 && d > 0);
    if (rows == 0) return NPUB_OK;
    NPUB_CHECK_ARG(x && gamma && G && ss);
    NPUB_CHECK_ARG(d % 32 == 0 && ldx % kVec == 0 && ldg % kVec == 0 && ldx >= d && ldg >= d && ss_ld >= rows);
    NPUB_CHECK_ARG(npub_aligned(x, 16) && npub_aligned(gamma, 16) && npub_aligned(G, 16));
    return launch_pdl(rms_parts_kernel, dim3(rows), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
                      reinterpret_cast<const __half*>(x), ldx, reinterpret_cast<const __half*>(gamma),
                      reinterpret_cast<__half*>(G), ldg, ss, ss_ld, d);
}

extern "C" int npub_swiglu(const void* g, int64_t ldg, const void* u, int64_t ldu, void* h, int64_t ldh, int rows,
                           int cols, void* stream) {
    NPUB_CHECK_ARG(rows >= 0 && cols >= 0);
    if (rows == 0 || cols == 0) return NPUB_OK;
    NPUB_CHECK_ARG(g && u && h && ldg >= cols && ldu >= cols && ldh >= cols);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const bool vec = cols % kVec == 0 && ldg % kVec == 0 && ldu % kVec == 0 && ldh % kVec == 0 &&
                     npub_aligned(g, 16) && npub_aligned(u, 16) && npub_aligned(h, 16);
    if (vec) {
        const int64_t work = (int64_t)rows * (cols / kVec);
        return launch_pdl(swiglu_vec_kernel, dim3(grid_for(work, 256)), dim3(256), 0, st,
                          reinterpret_cast<const __half*>(g), ldg, reinterpret_cast<const __half*>(u), ldu,
                          reinterpret_cast<__half*>(h), ldh, rows, cols);
    } else {
        const int64_t work = (int64_t)rows * cols;
        swiglu_scalar_kernel<<<grid_for(work, 256), 256, 0, st>>>(
            reinterpret_cast<const __half*>(g), ldg, reinterpret_cast<const __half*>(u), ldu,
            reinterpret_cast<__half*>(h), ldh, rows, cols);
    }
    return npub_internal_launch_status();
}

extern "C" int npub_softmax_rows(const void* s, void* p, int64_t ld, int64_t batch_stride, int batch, int rows,
                                 int cols, float scale, int causal_offset, int zero_full, void* stream) {
    NPUB_CHECK_ARG(batch >= 0 && rows >= 0 && cols >= 0);
    if (batch == 0 || rows == 0 || cols == 0) return NPUB_OK;
    NPUB_CHECK_ARG(s && p && ld >= cols && ld % kVec == 0 && npub_aligned(s, 16) && npub_aligned(p, 16));
    NPUB_CHECK_ARG(batch == 1 || (batch_stride >= ld * rows && batch_stride % kVec == 0));
    NPUB_CHECK_ARG(causal_offset >= NPUB_NO_CAUSAL);
    NPUB_CHECK_ARG((int64_t)batch * rows <= 0x7fffffffLL);
    NPUB_CHECK_ARG(cols <= 256 * 8 * 32);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int nb = batch * rows;
    const __half* sh = reinterpret_cast<const __half*>(s);
    __half* ph = reinterpret_cast<__half*>(p);
    const int nch = (cols + kVec - 1) / kVec;
    if (cols % kVec == 0 && nch <= 512) {
        const dim3 grid((unsigned)((nb + 7) / 8));
#define NPUB_SMW(C) softmax_warp_kernel<C><<<grid, 256, 0, st>>>(sh, ph, ld, batch_stride, rows, nb, cols, scale, \
                                                                  causal_offset, zero_full)
        if (nch <= 32) NPUB_SMW(1);
        else if (nch <= 64) NPUB_SMW(2);
        else if (nch <= 128) NPUB_SMW(4);
        else if (nch <= 256) NPUB_SMW(8);
        else NPUB_SMW(16);
#undef NPUB_SMW
        return npub_internal_launch_status();
    }
    if (nch <= 128)
        softmax_kernel<128, 1><<<nb, 128, 0, st>>>(sh, ph, ld, batch_stride, rows, cols, scale, causal_offset, zero_full);
    else if (nch <= 256)
        softmax_kernel<256, 1><<<nb, 256, 0, st>>>(sh, ph, ld, batch_stride, rows, cols, scale, causal_offset, zero_full);
    else if (nch <= 1024)
        softmax_kernel<256, 4><<<nb, 256, 0, st>>>(sh, ph, ld, batch_stride, rows, cols, scale, causal_offset, zero_full);
    else if (nch <= 4096)
        softmax_kernel<256, 16><<<nb, 256, 0, st>>>(sh, ph, ld, batch_stride, rows, cols, scale, causal_offset, zero_full);
    else
        softmax_kernel<256, 32><<<nb, 256, 0, st>>>(sh, ph, ld, batch_stride, rows, cols, scale, causal_offset, zero_full);
    return npub_internal_launch_status();
}

static int rope_impl(void* x, int64_t ldx, int tokens, int heads, int head_dim, const int32_t* positions, int pos0,
                     float theta, const float* inv_freq, void* stream) {
    NPUB_CHECK_ARG(tokens >= 0 && heads >= 0);
    if (tokens == 0 || heads == 0) return NPUB_OK;
    NPUB_CHECK_ARG(x && head_dim > 0 && head_dim % 2 == 0 && ldx >= (int64_t)heads * head_dim);
    NPUB_CHECK_ARG(inv_freq ? npub_aligned(inv_freq, 4) : theta > 0.0f);
    const float l2t = inv_freq ? 0.0f : log2f(theta);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (head_dim % 16 == 0 && head_dim <= 512 && ldx % 8 == 0 && npub_aligned(x, 16)) {
        return launch_pdl(rope_vec_kernel, dim3(tokens), dim3(128), 0, st, reinterpret_cast<__half*>(x), ldx, heads,
                          head_dim, positions, pos0, l2t, inv_freq);
    }
    const int64_t work = (int64_t)tokens * heads * (head_dim / 2);
    rope_kernel<<<grid_for(work, 256), 256, 0, st>>>(reinterpret_cast<__half*>(x), ldx, tokens, heads, head_dim,
                                                      positions, pos0, l2t, inv_freq);
    return npub_internal_launch_status();
}

extern "C" int npub_rope(void* x, int64_t ldx, int tokens, int heads, int head_dim, const int32_t* positions, int pos0,
                         float theta, void* stream) {
    return rope_impl(x, ldx, tokens, heads, head_dim, positions, pos0, theta, nullptr, stream);
}

extern "C" int npub_rope_freqs(void* x, int64_t ldx, int tokens, int heads, int head_dim, const int32_t* positions,
                               int pos0, const float* inv_freq, void* stream) {
    NPUB_CHECK_ARG(inv_freq);
    return rope_impl(x, ldx, tokens, heads, head_dim, positions, pos0, 0.0f, inv_freq, stream);
}

static int rope_kv_append_impl(void* qkv, int64_t ldx, int tokens, int q_heads, int kv_heads, int head_dim,
                               const int32_t* positions, float theta, const float* inv_freq, void* k_cache,
                               void* v_cache, int64_t cap, int32_t* lens, void* stream) {
    NPUB_CHECK_ARG(tokens >= 0 && q_heads >= 0 && kv_heads >= 0);
    if (tokens == 0) return NPUB_OK;
    NPUB_CHECK_ARG(qkv && positions && k_cache && v_cache && cap > 0);
    NPUB_CHECK_ARG(inv_freq ? npub_aligned(inv_freq, 4) : theta > 0.0f);
    NPUB_CHECK_ARG(head_dim % 16 == 0 && head_dim > 0 && head_dim <= 512);
    NPUB_CHECK_ARG(ldx >= (int64_t)(q_heads + 2 * kv_heads) * head_dim && ldx % 8 == 0);
    NPUB_CHECK_ARG(npub_aligned(qkv, 16) && npub_aligned(k_cache, 16) && npub_aligned(v_cache, 16));
    const int groups = (q_heads + 2 * kv_heads + 7) / 8;
    if (groups == 0) return NPUB_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    return launch_pdl(rope_kv_append_kernel, dim3(tokens, groups), dim3(64), 0, st, reinterpret_cast<__half*>(qkv),
                      ldx, q_heads, kv_heads, head_dim, 1, 8, positions, inv_freq ? 0.0f : log2f(theta), inv_freq,
                      reinterpret_cast<__half*>(k_cache), reinterpret_cast<__half*>(v_cache), cap, lens);
}

extern "C" int npub_rope_kv_append(void* qkv, int64_t ldx, int tokens, int q_heads, int kv_heads, int head_dim,
                                   const int32_t* positions, float theta, void* k_cache, void* v_cache, int64_t cap,
                                   int32_t* lens, void* stream) {
    return rope_kv_append_impl(qkv, ldx, tokens, q_heads, kv_heads, head_dim, positions, theta, nullptr, k_cache,
                               v_cache, cap, lens, stream);
}

extern "C" int npub_rope_kv_append_freqs(void* qkv, int64_t ldx, int tokens, int q_heads, int kv_heads, int head_dim,
                                         const int32_t* positions, const float* inv_freq, void* k_cache,
                                         void* v_cache, int64_t cap, int32_t* lens, void* stream) {
    NPUB_CHECK_ARG(inv_freq);
    return rope_kv_append_impl(qkv, ldx, tokens, q_heads, kv_heads, head_dim, positions, 0.0f, inv_freq, k_cache,
                               v_cache, cap, lens, stream);
}

static int rope_kv_store_impl(void* qkv, int64_t ldx, int tokens, int tokens_per_seq, int q_heads, int kv_heads,
                              int head_dim, const int32_t* positions, float theta, const float* inv_freq,
                              void* k_cache, void* v_cache, int64_t cap, void* stream) {
    NPUB_CHECK_ARG(tokens >= 0 && q_heads >= 0 && kv_heads >= 0);
    if (tokens == 0) return NPUB_OK;
    NPUB_CHECK_ARG(tokens_per_seq > 0 && tokens % tokens_per_seq == 0);
    NPUB_CHECK_ARG(qkv && positions && k_cache && v_cache && cap > 0);
    NPUB_CHECK_ARG(inv_freq ? npub_aligned(inv_freq, 4) : theta > 0.0f);
    NPUB_CHECK_ARG(head_dim % 16 == 0 && head_dim > 0 && head_dim <= 512);
    NPUB_CHECK_ARG(ldx >= (int64_t)(q_heads + 2 * kv_heads) * head_dim && ldx % 8 == 0);
    NPUB_CHECK_ARG(npub_aligned(qkv, 16) && npub_aligned(k_cache, 16) && npub_aligned(v_cache, 16));
    // a block rotates/stores up to 32 heads of one row (8 vectors of 8 per
    // head at head_dim 128: one per thread)
    const int hpb = 32;
    const int groups = (q_heads + 2 * kv_heads + hpb - 1) / hpb;
    if (groups == 0) return NPUB_OK;
    NPUB_CHECK_ARG(groups <= 65535);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    return launch_pdl(rope_kv_append_kernel, dim3(tokens, groups), dim3(256), 0, st, reinterpret_cast<__half*>(qkv),
                      ldx, q_heads, kv_heads, head_dim, tokens_per_seq, hpb, positions,
                      inv_freq ? 0.0f : log2f(theta), inv_freq, reinterpret_cast<__half*>(k_cache),
                      reinterpret_cast<__half*>(v_cache), cap, nullptr);
}

extern "C" int npub_rope_kv_store(void* qkv, int64_t ldx, int tokens, int tokens_per_seq, int q_heads, int kv_heads,
                                  int head_dim, const int32_t* positions, float theta, void* k_cache, void* v_cache,
                                  int64_t cap, void* stream) {
    return rope_kv_store_impl(qkv, ldx, tokens, tokens_per_seq, q_heads, kv_heads, head_dim, positions, theta, nullptr,
                              k_cache, v_cache, cap, stream);
}

extern "C" int npub_rope_kv_store_freqs(void* qkv, int64_t ldx, int tokens, int tokens_per_seq, int q_heads,
                                        int kv_heads, int head_dim, const int32_t* positions, const float* inv_freq,
                                        void* k_cache, void* v_cache, int64_t cap, void* stream) {
    NPUB_CHECK_ARG(inv_freq);
    return rope_kv_store_impl(qkv, ldx, tokens, tokens_per_seq, q_heads, kv_heads, head_dim, positions, 0.0f,
                              inv_freq, k_cache, v_cache, cap, stream);
}

// Host-side table of the per-frequency rates: theta^(-2i/hd) for i < hd/2,
// with the Llama-3 scaling of legalize.py:50-64 when factor > 0 (wavelengths
// above old_ctx/low divided by factor, below old_ctx/high kept, a smooth blend
// between), computed in double precision like the reference's numpy tables.
extern "C" int npub_rope_llama3_freqs(float* out, int head_dim, double theta, double factor, double low, double high,
                                      double old_ctx) {
    NPUB_CHECK_ARG(out && head_dim > 0 && head_dim % 2 == 0 && theta > 0.0);
    NPUB_CHECK_ARG(factor <= 0.0 || (high > low && low > 0.0 && old_ctx > 0.0));
    const double pi = 3.14159265358979323846;
    for (int i = 0; i < head_dim / 2; ++i) {
        const double f = std::pow(theta, -2.0 * i / head_dim);
        double r = f;
        if (factor > 0.0) {
            const double wl = 2.0 * pi / f;
            if (wl > old_ctx / low) {
                r = f / factor;
            } else if (wl >= old_ctx / high) {
                const double sm = (old_ctx / wl - low) / (high - low);
                r = (1.0 - sm) * f / factor + sm * f;
            }
        }
        out[i] = (float)r;
    }
    return NPUB_OK;
}

extern "C" int npub_quantize_w8(const float* W, int64_t ldw, int K, int N, int8_t* Wq, int64_t ldq, void* scale,
                                void* stream) {
    NPUB_CHECK_ARG(K >= 0 && N >= 0);
    if (K == 0 || N == 0) return NPUB_OK;
    NPUB_CHECK_ARG(W && Wq && scale && ldw >= N && ldq >= K);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    quantize_w8_kernel<<<(N + 31) / 32, 256, 0, st>>>(W, ldw, K, N, Wq, ldq, reinterpret_cast<__half*>(scale));
    return npub_internal_launch_status();
}

extern "C" int npub_add(const void* a, int64_t lda, const void* b, int64_t ldb, void* out, int64_t ldo, int rows,
                        int cols, void* stream) {
    NPUB_CHECK_ARG(rows >= 0 && cols >= 0);
    if (rows == 0 || cols == 0) return NPUB_OK;
    NPUB_CHECK_ARG(a && b && out && lda >= cols && ldb >= cols && ldo >= cols);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const bool vec = cols % kVec == 0 && lda % kVec == 0 && ldb % kVec == 0 && ldo % kVec == 0 && npub_aligned(a, 16) &&
                     npub_aligned(b, 16) && npub_aligned(out, 16);
    const __half* ah = reinterpret_cast<const __half*>(a);
    const __half* bh = reinterpret_cast<const __half*>(b);
    __half* oh = reinterpret_cast<__half*>(out);
    if (vec)
        return launch_pdl(add_vec_kernel, dim3(grid_for((int64_t)rows * (cols / kVec), 256)), dim3(256), 0, st, ah, lda,
                          bh, ldb, oh, ldo, rows, cols);
    else
        add_scalar_kernel<<<grid_for((int64_t)rows * cols, 256), 256, 0, st>>>(ah, lda, bh, ldb, oh, ldo, rows, cols);
    return npub_internal_launch_status();
}

extern "C" int npub_embed(const int32_t* ids, int n, const void* table, int64_t ldt, int vocab, int d, void* out,
                          int64_t ldo, void* stream) {
    NPUB_CHECK_ARG(n >= 0);
    if (n == 0) return NPUB_OK;
    NPUB_CHECK_ARG(ids && table && out && vocab > 0 && d > 0 && d % kVec == 0 && ldt >= d && ldo >= d);
    NPUB_CHECK_ARG(ldt % kVec == 0 && ldo % kVec == 0 && npub_aligned(table, 16) && npub_aligned(out, 16));
    return launch_pdl(embed_kernel, dim3(n), dim3(128), 0, reinterpret_cast<cudaStream_t>(stream), ids,
                      reinterpret_cast<const __half*>(table), ldt, vocab, d, reinterpret_cast<__half*>(out), ldo);
}

extern "C" int npub_argmax_rows(const void* x, int64_t ldx, int rows, int cols, int32_t* idx, float* val,
                                void* stream) {
    NPUB_CHECK_ARG(rows >= 0);
    if (rows == 0) return NPUB_OK;
    NPUB_CHECK_ARG(x && idx && cols > 0 && ldx >= cols);
    return launch_pdl(argmax_kernel, dim3(rows), dim3(512), 0, reinterpret_cast<cudaStream_t>(stream),
                      reinterpret_cast<const __half*>(x), ldx, cols, idx, val, (uint64_t*)nullptr, 0);
}

extern "C" int npub_argmax_keys(const void* x, int64_t ldx, int rows, int cols, int32_t index_offset, uint64_t* keys,
                                void* stream) {
    NPUB_CHECK_ARG(rows >= 0);
    if (rows == 0) return NPUB_OK;
    NPUB_CHECK_ARG(x && keys && cols > 0 && ldx >= cols && index_offset >= 0);
    NPUB_CHECK_ARG((int64_t)index_offset + cols <= 0x7fffffff && npub_aligned(keys, 8));
    return launch_pdl(argmax_kernel, dim3(rows), dim3(512), 0, reinterpret_cast<cudaStream_t>(stream),
                      reinterpret_cast<const __half*>(x), ldx, cols, (int32_t*)nullptr, (float*)nullptr, keys,
                      index_offset);
}

extern "C" int npub_select_keys(const uint64_t* keys, int ranks, int rows, int32_t* ids, void* stream) {
    NPUB_CHECK_ARG(rows >= 0 && ranks >= 0);
    if (rows == 0) return NPUB_OK;
    NPUB_CHECK_ARG(keys && ids && ranks > 0 && npub_aligned(keys, 8));
    return launch_pdl(select_keys_kernel, dim3((rows + 127) / 128), dim3(128), 0,
                      reinterpret_cast<cudaStream_t>(stream), keys, ranks, rows, ids);
}

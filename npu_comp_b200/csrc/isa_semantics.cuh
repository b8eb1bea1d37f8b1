// The NPU's elementwise instruction semantics (_poc/mysim.cpp:114-141) as the
// cmodel computes them on its x86-64 host, for the kernels that execute NPU
// instructions (isa_ops.cu, program.cu).
//
//  * float32, round to nearest, no contraction: mul-add and the matmul's
//    a += x * y are two roundings each;
//  * NaN results follow SSE: an operation with a NaN operand returns that
//    operand made quiet, and an invalid operation without NaN operands
//    (inf - inf, 0 * inf, 0 / 0, sqrt of a negative) returns the "indefinite"
//    NaN 0xFFC00000, whose sign the fp16 store keeps (0xFE00).  When both
//    operands are NaN the one the compiled cmodel holds in the destination
//    register wins; measured on the reference simulator built here: the left
//    operand of a op b, the product in mul-add (pout + a * b), the running sum
//    in the matmul (acc += x * y), and in the activation x * x * sigmoid(x)
//    the sigmoid after a matmul, x * x after an elementwise matrix op.  CUDA's
//    own NaN is the positive 0x7FFFFFFF, so every NaN result is replaced here;
//  * conversions to integer are cvttss2si: truncation, and INT64_MIN (or
//    INT32_MIN) for NaN and out-of-range values;
//  * exp is CUDA's expf (a few float32 ulps from the host libm).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace npub {
namespace isa {

__device__ __forceinline__ float quiet(float x) { return __uint_as_float(__float_as_uint(x) | 0x00400000u); }

// The SSE result of a binary operation x (op) y whose IEEE value is r.
__device__ __forceinline__ float sse2(float r, float x, float y) {
    if (!isnan(r)) return r;
    if (isnan(x)) return quiet(x);
    if (isnan(y)) return quiet(y);
    return __uint_as_float(0xFFC00000u);
}
// The same for a unary operation of x.
__device__ __forceinline__ float sse1(float r, float x) {
    if (!isnan(r)) return r;
    if (isnan(x)) return quiet(x);
    return __uint_as_float(0xFFC00000u);
}

__device__ __forceinline__ float add(float x, float y) { return sse2(__fadd_rn(x, y), x, y); }
__device__ __forceinline__ float sub(float x, float y) { return sse2(__fsub_rn(x, y), x, y); }
__device__ __forceinline__ float mul(float x, float y) { return sse2(__fmul_rn(x, y), x, y); }
__device__ __forceinline__ float div(float x, float y) { return sse2(__fdiv_rn(x, y), x, y); }

__device__ __forceinline__ long long to_i64(float a) {
    if (!(fabsf(a) < 9.2233720368547758e18f)) return (long long)0x8000000000000000ULL;
    return __float2ll_rz(a);
}
__device__ __forceinline__ int to_i32(float a) {
    if (!(fabsf(a) < 2147483648.0f)) return (int)0x80000000u;
    return __float2int_rz(a);
}
// Exact 2^s in float32 (0 below the subnormal range, inf above 127), as powf(2, s).
__device__ __forceinline__ float exp2_int(int s) {
    if (s > 127) return __int_as_float(0x7f800000);
    if (s >= -126) return __int_as_float((s + 127) << 23);
    if (s >= -149) return __int_as_float(1 << (s + 149));
    return 0.0f;
}
__device__ __forceinline__ float expf_host(float x) { return sse1(expf(x), x); }
// -x as the host computes it: a sign flip, NaN included.
__device__ __forceinline__ float neg(float x) { return __uint_as_float(__float_as_uint(x) ^ 0x80000000u); }
// act(x) = x * x * sigmoid(x), sigmoid(x) = 1 / (1 + exp(-x)) (mysim.cpp:39-40);
// sigmoid_first: which factor's NaN wins when both are NaN (see above).
__device__ __forceinline__ float act(float x, bool sigmoid_first) {
    const float s = div(1.0f, add(1.0f, expf_host(neg(x))));
    const float xx = mul(x, x);
    return sigmoid_first ? mul(s, xx) : mul(xx, s);
}

// One element of a compute instruction: a from PE input 1, b the second
// operand (PE input 2 in vector mode, else the immediate), prev the previous
// PE output (read by mul-add 0x0C).
__device__ __forceinline__ float elem_op(uint32_t w, float a, float b, float prev) {
    const uint32_t op = w & 0xFFu;
    const int mode = (int)((w >> 30) & 3u);
    const bool matrix = op >= 0x40u && op <= 0x43u;
    const int cst = (int)((w >> 8) & 0xFFFFu);
    float r = a;
    switch (op) {
        case 0x01: case 0x40: r = add(a, b); break;
        case 0x02: case 0x41: r = sub(a, b); break;
        case 0x0A: case 0x42: r = mul(a, b); break;
        case 0x0B: r = div(a, b); break;
        case 0x0C: r = add(mul(a, b), prev); break;
        case 0x0D: case 0x43: r = b; break;
        case 0x0E: r = sse1(__fsqrt_rn(a), a); break;
        case 0x0F: r = expf_host(a); break;
        case 0x11: r = (a == b) ? 1.0f : 0.0f; break;
        case 0x12: r = ((w >> 28) & 1u) ? ((a > b) ? a : b) : ((a < b) ? a : b); break;
        case 0x13: r = __ll2float_rn(to_i64(a)); break;
        case 0x09: {
            short s = (short)cst;
            if (mode == 2) s = (short)to_i32(b);
            r = mul(a, exp2_int((int)s));
        } break;
        case 0x08: {
            const long long ia = to_i64(a), ib = to_i64(b);
            switch ((w >> 27) & 7u) {
                case 0: r = __ll2float_rn(ia & ib); break;
                case 1: r = __ll2float_rn(ia | ib); break;
                case 2: r = __ll2float_rn(~ia); break;
                case 3: r = __ll2float_rn(ia ^ ib); break;
                case 4: r = __ll2float_rn(~(ia & ib)); break;
                case 5: r = __ll2float_rn(~(ia | ib)); break;
                default: break;
            }
        } break;
        default: break;
    }
    if (((w >> 29) & 1u) && matrix) r = act(r, false);
    return r;
}

// The cmodel's fp16 store bits (mysim.cpp:19-38): round to nearest even,
// overflow to inf, NaN -> sign | 0x7C00 | 0x200.
__device__ __forceinline__ uint16_t f16_bits(float v) {
    const uint32_t u = __float_as_uint(v);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x7fffffu)) return (uint16_t)(((u >> 16) & 0x8000u) | 0x7E00u);
    return __half_as_ushort(__float2half_rn(v));
}
// fp16 word -> float32 as the cmodel widens G-buffer words (mysim.cpp:28-35):
// exact for numbers; a NaN keeps its sign and payload (sign | 0x7F800000 |
// mantissa << 13), which the hardware conversion would replace by its
// canonical positive NaN.
__device__ __forceinline__ float h2f(uint16_t h) {
    if ((h & 0x7C00u) == 0x7C00u && (h & 0x3FFu))
        return __uint_as_float(((uint32_t)(h & 0x8000u) << 16) | 0x7F800000u | ((uint32_t)(h & 0x3FFu) << 13));
    return __half2float(__ushort_as_half(h));
}
// The stored value back as float32 (what the G-buffer holds after a save).
__device__ __forceinline__ float round_f16(float v) { return h2f(f16_bits(v)); }

}  // namespace isa
}  // namespace npub

// The NPU's elementwise instruction semantics on sm_100a (_poc/mysim.cpp:114-141)
// and its fp16 store rounding (mysim.cpp:19-38).
//
// The per-element semantics are those of isa_semantics.cuh: the cmodel's bits
// (float32 without contraction, SSE NaN results, x86-64 integer conversions)
// except exp and the matrix activation x^2*sigmoid(x), which use CUDA's expf
// and agree within a few float32 ulps.
#include "common.cuh"
#include "isa_semantics.cuh"

namespace npub {

__global__ void isa_vector_kernel(uint32_t w, const float* __restrict__ in1, const float* __restrict__ in2,
                                  const float* __restrict__ prev, float* __restrict__ out, int64_t n) {
    const int mode = (int)((w >> 30) & 3u);
    const int cst = (int)((w >> 8) & 0xFFFFu);
    const bool uses_prev = (w & 0xFFu) == 0x0Cu;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float b = (mode == 2) ? in2[i] : (float)cst;
        out[i] = isa::elem_op(w, in1[i], b, uses_prev ? prev[i] : 0.0f);
    }
}

// fp32 -> fp16 with the cmodel's conversion (RNE; NaN keeps its sign and
// becomes the quiet pattern 0x7E00).
__global__ void f32_to_f16_kernel(const float* __restrict__ x, uint16_t* __restrict__ y, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        y[i] = isa::f16_bits(x[i]);
    }
}

__global__ void f16_to_f32_kernel(const uint16_t* __restrict__ x, float* __restrict__ y, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = isa::h2f(x[i]);
}

static int blocks_for(int64_t n) {
    int64_t b = (n + 255) / 256;
    if (b > 148 * 32) b = 148 * 32;
    return (int)(b < 1 ? 1 : b);
}

}  // namespace npub

using namespace npub;

extern "C" int npub_isa_vector(uint32_t word, const float* in1, const float* in2, const float* prev_out, float* out,
                               int64_t n, void* stream) {
    NPUB_CHECK_ARG(n >= 0);
    if (n == 0) return NPUB_OK;
    const uint32_t op = word & 0xFFu;
    const int mode = (int)((word >> 30) & 3u);
    const bool supported = (op >= 0x01 && op <= 0x02) || (op >= 0x08 && op <= 0x0F) || (op >= 0x11 && op <= 0x13) ||
                           (op >= 0x40 && op <= 0x43);
    if (!supported || (op == 0x42 && mode == 2)) return NPUB_ERR_UNSUPPORTED;
    NPUB_CHECK_ARG(in1 && out);
    NPUB_CHECK_ARG(mode != 2 || in2);
    NPUB_CHECK_ARG(op != 0x0C || prev_out);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    isa_vector_kernel<<<blocks_for(n), 256, 0, st>>>(word, in1, in2, prev_out, out, n);
    return npub_internal_launch_status();
}

extern "C" int npub_f32_to_f16(const float* x, uint16_t* y, int64_t n, void* stream) {
    NPUB_CHECK_ARG(n >= 0);
    if (n == 0) return NPUB_OK;
    NPUB_CHECK_ARG(x && y);
    f32_to_f16_kernel<<<blocks_for(n), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(x, y, n);
    return npub_internal_launch_status();
}

extern "C" int npub_f16_to_f32(const uint16_t* x, float* y, int64_t n, void* stream) {
    NPUB_CHECK_ARG(n >= 0);
    if (n == 0) return NPUB_OK;
    NPUB_CHECK_ARG(x && y);
    f16_to_f32_kernel<<<blocks_for(n), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(x, y, n);
    return npub_internal_launch_status();
}

// npub_w8a16_gemm_noalloc: the W8A16 matmul for callers that cannot allocate
// device memory.
//
// Some hosts of this library own every byte of device memory and forbid other
// allocators (a plugin living inside another runtime's memory pool), some have
// no device allocator at all (a plain C or ctypes caller without a framework),
// and some run where cudaMalloc is not allowed or would stall the device (a
// latency-critical decode loop with a fixed memory budget).  Such callers can
// still pass their inputs and outputs, but not the split-K workspace that
// npub_w8a16_gemm asks for.  This entry point takes that scratch from a
// fixed-size array in the library's own device globals instead.
//
// The array lives in every device that loads the library until the process
// exits.  Every call shares it and it keeps the last call's contents.  Its
// first kSkinnyCounterBytes hold the tile counters of the few-token (M <= 64)
// kernel, which start at zero (the array is zero-initialised when the module
// loads) and which every completed call leaves at zero; nothing else is ever
// written there.  A call in which a bounded wait gave up (the device error
// word set, NPUB_ERR_DEVICE_TIMEOUT from npub_device_error) may leave counts
// behind; npub_device_error(1) re-zeroes them along with the error word.  The rest holds split-K partials, fully overwritten before
// they are read.  Calls that overlap on the GPU (different streams, or
// different host threads on the same device) race on the array.
#include "common.cuh"
#include "gemm_w8a16_skinny.h"

#include <mutex>

// File-scope scratch: NPUB_NOALLOC_SCRATCH_BYTES per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[NPUB_NOALLOC_SCRATCH_BYTES];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64];

// Device address of g_noalloc_scratch for the current device.  In host code
// the array's name is only a host-side stand-in, so the address is looked up
// once per device, with that device current, and cached.  The cache assumes
// the module stays loaded: the library must not be used across a
// cudaDeviceReset (which unloads the module and frees the array).
static int noalloc_scratch(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        npub_internal_set_cuda_error(e);
        return NPUB_ERR_CUDA;
    }
    if (dev < 0 || dev >= 64) return NPUB_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            npub_internal_set_cuda_error(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
            return NPUB_ERR_CUDA;
        }
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return NPUB_OK;
}

int npub_internal_noalloc_reset() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        npub_internal_set_cuda_error(e);
        return NPUB_ERR_CUDA;
    }
    if (dev < 0 || dev >= 64) return NPUB_OK;
    void* p = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        p = g_noalloc_ptr[dev];
    }
    if (!p) return NPUB_OK;  // never used on this device: the counters are still zero
    // cudaMemset writes the counters in place; nothing is allocated
    e = cudaMemset(p, 0, npub::kSkinnyCounterBytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        npub_internal_set_cuda_error(e);
        return NPUB_ERR_CUDA;
    }
    return NPUB_OK;
}

extern "C" int npub_w8a16_gemm_noalloc(const void* A, int64_t lda, const int8_t* Wq, int64_t ldw, const void* scale,
                                       void* C, int64_t ldc, const void* R, int64_t ldr, int M, int N, int K,
                                       float alpha, void* stream) {
    if (M < 0 || N < 0 || K < 0) return NPUB_ERR_INVALID_ARG;
    // Every W8A16 workspace layout starts with the counter region, so all
    // calls can share the array from its start.
    const size_t need = npub_w8a16_gemm_workspace(M, N, K);
    if (need > (size_t)NPUB_NOALLOC_SCRATCH_BYTES) return NPUB_ERR_SCRATCH_LIMIT;
    void* ws = nullptr;
    if (need > 0) {
        const int rc = noalloc_scratch(&ws);
        if (rc != NPUB_OK) return rc;
    }
    return npub_w8a16_gemm(A, lda, Wq, ldw, scale, C, ldc, R, ldr, M, N, K, alpha, ws, need, stream);
}

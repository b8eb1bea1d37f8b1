// Library-wide C ABI pieces: version, status strings, CUDA error capture and
// the per-device error word that kernels set when a bounded wait gives up.
#include "common.cuh"

#include <atomic>
#include <cstdlib>

// One int per device context (module globals are instantiated per device).
__device__ int g_npub_device_error;

static thread_local int t_last_cuda_error = 0;
static std::atomic<unsigned long long> g_launches{0};

void npub_internal_set_cuda_error(cudaError_t e) { t_last_cuda_error = (int)e; }

bool npub_internal_pdl_enabled() {
    static const bool on = [] {
        const char* v = getenv("NPUB_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

int npub_internal_launch_status() {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        t_last_cuda_error = (int)e;
        return NPUB_ERR_CUDA;
    }
    return NPUB_OK;
}

uint64_t npub_internal_wait_limit_ns() {
    static const uint64_t ns = [] {
        const char* v = getenv("NPUB_WAIT_LIMIT_MS");
        long ms = v ? strtol(v, nullptr, 10) : 2000;
        if (ms < 1) ms = 1;
        if (ms > 60000) ms = 60000;
        return (uint64_t)ms * 1000000ull;
    }();
    return ns;
}

bool npub_internal_l2_evict_first() {
    static const bool on = [] {
        const char* v = getenv("NPUB_L2_EVICT_FIRST");
        return !(v && v[0] == '0');
    }();
    return on;
}

int* npub_internal_device_error_word() {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_npub_device_error) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return reinterpret_cast<int*>(p);
}

extern "C" int npub_version(void) { return 10000; }

extern "C" const char* npub_strerror(int status) {
    switch (status) {
        case NPUB_OK: return "ok";
        case NPUB_ERR_INVALID_ARG: return "invalid argument (shape, stride, alignment or null pointer)";
        case NPUB_ERR_UNSUPPORTED: return "unsupported configuration";
        case NPUB_ERR_CUDA: return "CUDA error";
        case NPUB_ERR_WORKSPACE: return "workspace missing or too small";
        case NPUB_ERR_DEVICE_TIMEOUT: return "a device-side wait timed out";
        case NPUB_ERR_NO_DEVICE: return "no sm_100 device";
        case NPUB_ERR_SCRATCH_LIMIT:
            return "request needs more split-K scratch than the allocation-free entry point holds "
                   "(NPUB_NOALLOC_SCRATCH_BYTES); use npub_w8a16_gemm with a workspace";
        default: return "unknown status";
    }
}

extern "C" int npub_last_cuda_error(void) { return t_last_cuda_error; }

extern "C" unsigned long long npub_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" int npub_device_error(int clear) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        t_last_cuda_error = (int)e;
        return NPUB_ERR_CUDA;
    }
    int v = 0;
    e = cudaMemcpyFromSymbol(&v, g_npub_device_error, sizeof(int));
    if (e != cudaSuccess) {
        t_last_cuda_error = (int)e;
        return NPUB_ERR_CUDA;
    }
    if (clear) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_npub_device_error, &zero, sizeof(int));
        if (e != cudaSuccess) {
            t_last_cuda_error = (int)e;
            return NPUB_ERR_CUDA;
        }
        // A stream-K call whose wait gave up may have left counts in its tile
        // counters; the library's own (allocation-free) scratch is reset
        // here, a caller's workspace by its owner.
        int rc = npub_internal_noalloc_reset();
        if (rc != NPUB_OK) return rc;
        rc = npub_internal_decode_flags_reset();  // the decode attention finishers' piece flags
        if (rc != NPUB_OK) return rc;
    }
    return v;
}

// One-shot all-reduce over NVLink peer memory for the small messages of
// tensor-parallel decode (the two per-layer reductions of a [batch, d] fp16
// activation under the Llama layer's TP sharding).  NCCL stays in use
// for large messages (prefill), where its bandwidth-optimal algorithms win;
// at a few hundred KB its per-call latency inside a CUDA graph (21 us on 2
// B200s, 36 us on 8, measured) is most of a decode layer.
//
// Each rank owns one IPC-shareable allocation:
//   [data: 2 x max_bytes][flags: world x kMaxBlocks uint32][epochs: kMaxBlocks uint32]
// and maps every peer's allocation (cudaIpcOpenMemHandle).  Block b always
// owns the same region of each half (max_bytes / kCommMaxBlocks), whatever
// the message size, so only the blocks b of the ranks ever touch it.  A call
// with block epoch e (per-block counters, so graphs can replay the call) uses
// half e & 1:
//   1. block b copies its slice of the input into its region of its own half,
//   2. publishes e to flags[rank][b] of every rank (system-scope release),
//   3. waits until flags[r][b] >= e for every r (bounded; acquire),
//   4. sums slice b of every rank's half in rank order 0..world-1 in fp32 and
//      writes fp16 (the same bits on every rank),
//   5. stores its epoch.
// Block b only ever waits for the blocks b of its peers, each on its own GPU,
// so no two blocks of one GPU wait on each other.  Reusing a half two calls
// later is safe: passing step 3 of call e + 1 means every peer has finished
// call e.
#include "common.cuh"
#include "gemm_w8a16_skinny.h"

#include <cstring>
#include <mutex>

namespace npub {

constexpr int kCommMaxRanks = 8;
constexpr int kCommMaxBlocks = 256;  // fixed regions: 4 KB each at max_bytes = 1 MB
constexpr int kCommThreads = 256;

struct CommDev {
    __half* data[kCommMaxRanks];     // each rank's data area (2 halves)
    uint32_t* flags[kCommMaxRanks];  // each rank's flags [world][kCommMaxBlocks]
    uint32_t* epochs;                // this rank's per-block epochs
    int world, rank;
    int64_t half_elems;              // elements per data half
};

struct Comm {
    int world = 0, rank = 0, dev = 0;
    size_t max_bytes = 0, total = 0;
    void* base = nullptr;                  // own allocation
    void* peer_base[kCommMaxRanks] = {};   // opened peer allocations (own: base)
    CommDev d{};
};

// n elements (multiple of 8), 16-byte aligned in and out.
// Optional RMSNorm inputs for the next projection (nrm.resid != NULL): out =
// fp16(fp16(sum) + resid) -- the residual add of the separate RMSNorm -- and
// G = fp16(out * gamma[col]), ss[(col / 32) * ss_ld + row] = sum over the 32
// columns of out^2, for a [rows, d] message (npub_w8a16_gemm_rms consumes them).
struct CommNorm {
    const __half* resid;
    const __half* gamma;
    __half* G;
    float* ss;
    int64_t ss_ld;
    int d;
};

__global__ void __launch_bounds__(kCommThreads) allreduce_oneshot_kernel(const CommDev c, const __half* in,
                                                                        __half* out, int64_t n, int* err,
                                                                        uint64_t limit_ns, const CommNorm nrm) {
    pdl_trigger();
    pdl_wait();
    __shared__ int ok_s;
    const int b = blockIdx.x;
    const uint32_t e = c.epochs[b] + 1u;
    const int64_t nv = n / 8;                                  // 16-byte vectors
    const int64_t per = c.half_elems / 8 / kCommMaxBlocks;     // the block's fixed region
    const int64_t v0 = (int64_t)b * per, v1 = min(nv, v0 + per);
    const int64_t off = (int64_t)(e & 1u) * c.half_elems;
    // 1. own slice into the own half
    uint4* mine = reinterpret_cast<uint4*>(c.data[c.rank] + off);
    const uint4* src = reinterpret_cast<const uint4*>(in);
    for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x) mine[i] = src[i];
    __threadfence_system();
    __syncthreads();
    // 2. publish, 3. wait for every rank's block b
    if (threadIdx.x < c.world) st_release_sys(c.flags[threadIdx.x] + c.rank * kCommMaxBlocks + b, e);
    if (threadIdx.x == 0) ok_s = 1;
    __syncthreads();
    if (threadIdx.x < c.world) {
        const uint32_t* f = c.flags[c.rank] + threadIdx.x * kCommMaxBlocks + b;
        bool ok = ld_acquire_sys(f) >= e;
        if (!ok) {
            const uint64_t t0 = globaltimer_ns();
            for (uint32_t it = 1;; ++it) {
                if (ld_acquire_sys(f) >= e) {
                    ok = true;
                    break;
                }
                if ((it & 1023u) == 0 && globaltimer_ns() - t0 > limit_ns) break;
            }
        }
        if (!ok) {
            ok_s = 0;
            if (err) atomicCAS(err, 0, 0x501);
        }
    }
    cta_sync_divergent();  // lanes < world spun alone
    if (ok_s && nrm.resid) {
        // 4'. the sum, the residual add and the next RMSNorm's inputs; a warp
        // walks 32 consecutive vectors per step (4 lanes = 32 columns)
        const int lane = threadIdx.x & 31;
        for (int64_t base = v0 + (threadIdx.x & ~31); base < v1; base += blockDim.x) {
            const int64_t i = base + lane;
            const bool valid = i < v1;
            float h[8], sq = 0.0f;
            if (valid) {
                uint4 u[kCommMaxRanks];
#pragma unroll
                for (int r = 0; r < kCommMaxRanks; ++r)
                    if (r < c.world) u[r] = ld_relaxed_sys_v4(reinterpret_cast<const uint4*>(c.data[r] + off) + i);
                float acc[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) acc[k] = 0.0f;
#pragma unroll
                for (int r = 0; r < kCommMaxRanks; ++r) {
                    if (r >= c.world) break;
                    const __half2* h2 = reinterpret_cast<const __half2*>(&u[r]);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float2 f = __half22float2(h2[k]);
                        acc[2 * k] += f.x;
                        acc[2 * k + 1] += f.y;
                    }
                }
                const uint4 rv = reinterpret_cast<const uint4*>(nrm.resid)[i];
                const __half* rh = reinterpret_cast<const __half*>(&rv);
                uint4 o, g;
                __half* oh = reinterpret_cast<__half*>(&o);
                __half* gh = reinterpret_cast<__half*>(&g);
                const int64_t col = (i * 8) % nrm.d;
                const uint4 gv = *reinterpret_cast<const uint4*>(nrm.gamma + col);
                const __half* gm = reinterpret_cast<const __half*>(&gv);
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    oh[k] = __float2half_rn(__half2float(__float2half_rn(acc[k])) + __half2float(rh[k]));
                    h[k] = __half2float(oh[k]);
                    gh[k] = __float2half_rn(h[k] * __half2float(gm[k]));
                    sq += h[k] * h[k];
                }
                reinterpret_cast<uint4*>(out)[i] = o;
                reinterpret_cast<uint4*>(nrm.G)[i] = g;
            }
            sq += __shfl_xor_sync(0xffffffffu, sq, 1);
            sq += __shfl_xor_sync(0xffffffffu, sq, 2);
            if (valid && (lane & 3) == 0) {
                const int64_t e = i * 8;
                nrm.ss[(e % nrm.d) / 32 * nrm.ss_ld + e / nrm.d] = sq;
            }
        }
    } else if (ok_s) {
        // 4. sum slice b over the ranks, in rank order
        for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x) {
            // every rank's vector in flight before the first is added
            uint4 u[kCommMaxRanks];
#pragma unroll
            for (int r = 0; r < kCommMaxRanks; ++r)
                if (r < c.world) u[r] = ld_relaxed_sys_v4(reinterpret_cast<const uint4*>(c.data[r] + off) + i);
            float acc[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[k] = 0.0f;
#pragma unroll
            for (int r = 0; r < kCommMaxRanks; ++r) {
                if (r >= c.world) break;
                const __half2* h2 = reinterpret_cast<const __half2*>(&u[r]);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float2 f = __half22float2(h2[k]);
                    acc[2 * k] += f.x;
                    acc[2 * k + 1] += f.y;
                }
            }
            uint4 o;
            __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
            for (int k = 0; k < 4; ++k) oh[k] = __floats2half2_rn(acc[2 * k], acc[2 * k + 1]);
            reinterpret_cast<uint4*>(out)[i] = o;
        }
    }
    __syncthreads();
    // 5. the epoch advances even after a failed wait, so the ranks stay in step
    if (threadIdx.x == 0) c.epochs[b] = e;
}

}  // namespace npub

using namespace npub;

extern "C" size_t npub_comm_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int npub_comm_create(int world, int rank, size_t max_bytes, void** comm_out, void* handle_out) {
    NPUB_CHECK_ARG(comm_out && handle_out && world >= 1 && world <= kCommMaxRanks && rank >= 0 && rank < world);
    NPUB_CHECK_ARG(max_bytes > 0 && max_bytes % (16 * kCommMaxBlocks) == 0);
    Comm* c = new Comm();
    c->world = world;
    c->rank = rank;
    c->max_bytes = max_bytes;
    NPUB_CUDA_TRY(cudaGetDevice(&c->dev));
    const size_t flags_bytes = (size_t)kCommMaxRanks * kCommMaxBlocks * sizeof(uint32_t);
    const size_t epoch_bytes = (size_t)kCommMaxBlocks * sizeof(uint32_t);
    c->total = 2 * max_bytes + flags_bytes + epoch_bytes;
    cudaError_t e = cudaMalloc(&c->base, c->total);
    if (e == cudaSuccess) e = cudaMemset(c->base, 0, c->total);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->base);
    if (e != cudaSuccess) {
        if (c->base) cudaFree(c->base);
        delete c;
        npub_internal_set_cuda_error(e);
        return NPUB_ERR_CUDA;
    }
    memcpy(handle_out, &h, sizeof(h));
    *comm_out = c;
    return NPUB_OK;
}

extern "C" int npub_comm_open(void* comm, const void* all_handles) {
    NPUB_CHECK_ARG(comm && all_handles);
    Comm* c = reinterpret_cast<Comm*>(comm);
    const uint8_t* hs = reinterpret_cast<const uint8_t*>(all_handles);
    for (int r = 0; r < c->world; ++r) {
        if (r == c->rank) {
            c->peer_base[r] = c->base;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, hs + (size_t)r * sizeof(h), sizeof(h));
        void* p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            npub_internal_set_cuda_error(e);
            return NPUB_ERR_CUDA;
        }
        c->peer_base[r] = p;
    }
    CommDev& d = c->d;
    memset(&d, 0, sizeof(d));
    d.world = c->world;
    d.rank = c->rank;
    d.half_elems = (int64_t)(c->max_bytes / sizeof(__half));
    for (int r = 0; r < c->world; ++r) {
        uint8_t* b = reinterpret_cast<uint8_t*>(c->peer_base[r]);
        d.data[r] = reinterpret_cast<__half*>(b);
        d.flags[r] = reinterpret_cast<uint32_t*>(b + 2 * c->max_bytes);
    }
    d.epochs = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(c->base) + 2 * c->max_bytes +
                                           (size_t)kCommMaxRanks * kCommMaxBlocks * sizeof(uint32_t));
    return NPUB_OK;
}

static int allreduce_launch(void* comm, const void* in, void* out, int64_t n, const CommNorm& nrm, void* stream) {
    NPUB_CHECK_ARG(comm && n >= 0);
    if (n == 0) return NPUB_OK;
    Comm* c = reinterpret_cast<Comm*>(comm);
    NPUB_CHECK_ARG(in && out && n % 8 == 0 && (size_t)n * sizeof(__half) <= c->max_bytes);
    NPUB_CHECK_ARG(npub_aligned(in, 16) && npub_aligned(out, 16));
    NPUB_CHECK_ARG(c->d.data[0] != nullptr);  // npub_comm_open done
    // one block per fixed region the message reaches
    const int64_t region = (int64_t)(c->max_bytes / sizeof(__half)) / kCommMaxBlocks;
    if (nrm.resid) NPUB_CHECK_ARG(region % 32 == 0);  // a block's slice is whole 32-column chunks
    const int64_t blocks = (n + region - 1) / region;
    return launch_pdl(allreduce_oneshot_kernel, dim3((unsigned)blocks), dim3(kCommThreads), 0,
                      reinterpret_cast<cudaStream_t>(stream), c->d, reinterpret_cast<const __half*>(in),
                      reinterpret_cast<__half*>(out), n, npub_internal_device_error_word(),
                      npub_internal_wait_limit_ns(), nrm);
}

extern "C" int npub_allreduce_f16(void* comm, const void* in, void* out, int64_t n, void* stream) {
    CommNorm nrm;
    memset(&nrm, 0, sizeof(nrm));
    return allreduce_launch(comm, in, out, n, nrm, stream);
}

extern "C" int npub_allreduce_f16_rms(void* comm, const void* in, void* out, int rows, int d, const void* residual,
                                      const void* gamma, void* G, float* ss, int64_t ss_ld, void* stream) {
    NPUB_CHECK_ARG(rows >= 0 && d > 0 && d % 32 == 0);
    if (rows == 0) return NPUB_OK;
    NPUB_CHECK_ARG(residual && gamma && G && ss && ss_ld >= rows);
    NPUB_CHECK_ARG(npub_aligned(residual, 16) && npub_aligned(gamma, 16) && npub_aligned(G, 16));
    CommNorm nrm;
    nrm.resid = reinterpret_cast<const __half*>(residual);
    nrm.gamma = reinterpret_cast<const __half*>(gamma);
    nrm.G = reinterpret_cast<__half*>(G);
    nrm.ss = ss;
    nrm.ss_ld = ss_ld;
    nrm.d = d;
    return allreduce_launch(comm, in, out, (int64_t)rows * d, nrm, stream);
}

extern "C" int npub_comm_destroy(void* comm) {
    if (!comm) return NPUB_OK;
    Comm* c = reinterpret_cast<Comm*>(comm);
    int dev0 = 0;
    cudaGetDevice(&dev0);
    cudaSetDevice(c->dev);
    for (int r = 0; r < c->world; ++r)
        if (r != c->rank && c->peer_base[r]) cudaIpcCloseMemHandle(c->peer_base[r]);
    if (c->base) cudaFree(c->base);
    cudaSetDevice(dev0);
    delete c;
    return NPUB_OK;
}

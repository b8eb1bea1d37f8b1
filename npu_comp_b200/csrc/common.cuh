// Shared helpers for the sm_100a kernels of libnpub: status codes, argument
// checks, PTX wrappers for mbarriers, TMA, tcgen05 and the device error word.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "npub.h"

#define NPUB_CHECK_ARG(cond) \
    do {                     \
        if (!(cond)) return NPUB_ERR_INVALID_ARG; \
    } while (0)

#define NPUB_CUDA_TRY(expr)                                   \
    do {                                                      \
        cudaError_t e_ = (expr);                              \
        if (e_ != cudaSuccess) {                              \
            npub_internal_set_cuda_error(e_);                 \
            return NPUB_ERR_CUDA;                             \
        }                                                     \
    } while (0)

// Records the last CUDA error for npub_strerror/npub_last_cuda_error.
void npub_internal_set_cuda_error(cudaError_t e);
// Status after a kernel launch: checks cudaGetLastError.
int npub_internal_launch_status();
// Device error word used by bounded waits (one per device, zero-initialised).
int* npub_internal_device_error_word();
// Limit of the waits on other CTAs' or other ranks' progress (stream-K tile
// pieces, peer flags of the all-reduces): NPUB_WAIT_LIMIT_MS in the
// environment when the library loads (1 ms .. 60 s), else 2 s.
uint64_t npub_internal_wait_limit_ns();
// Streamed-once loads (decode weights, K/V stages) carry an evict-first L2
// policy unless NPUB_L2_EVICT_FIRST=0 is set in the environment.
bool npub_internal_l2_evict_first();
// Re-zeroes the allocation-free entry point's tile counters on the current
// device (after a wait gave up, they may hold counts of the aborted call).
int npub_internal_noalloc_reset();
// Re-zeroes the persistent decode attention's piece flags on the current device.
int npub_internal_decode_flags_reset();

static inline bool npub_aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Programmatic dependent launch.  Kernels launched through launch_pdl may be
// scheduled while the previous kernel on the stream is still running: each
// one calls pdl_trigger() on entry (so that its own successor may be
// scheduled early) and pdl_wait() before it reads or writes any memory that
// earlier kernels use; set-up that touches no such memory (barrier init,
// tensor-memory allocation, L2 prefetch of operands) overlaps the previous
// kernel's tail.  NPUB_PDL=0 in the environment launches them normally.
bool npub_internal_pdl_enabled();

template <typename... KArgs, typename... Args>
static inline int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = npub_internal_pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
    if (e != cudaSuccess) {
        npub_internal_set_cuda_error(e);
        return NPUB_ERR_CUDA;
    }
    return npub_internal_launch_status();
}

// ----------------------------------------------------------------- device side
namespace npub {

__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait on an mbarrier phase.  Gives up after `limit_ns` of wall time
// or as soon as `*abort` is set by another role of the CTA; returns false
// then, so every spin in these kernels ends.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort,
                                                  uint64_t limit_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0) {
            if (*abort) return false;
            if (globaltimer_ns() - t0 > limit_ns) return false;
        }
    }
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* m) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// ---- system-scope (peer GPU) flags and loads for the NVLink collectives
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Relaxed system-scope load: coherent with the peers' writes (no stale
// cache line) and, unlike a volatile load, free to overlap with the others.
__device__ __forceinline__ uint4 ld_relaxed_sys_v4(const void* p) {
    uint4 v;
    asm volatile("ld.relaxed.sys.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// L2 prefetch of one 3-D tile of a tensor map (no shared memory written).
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* m, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                     reinterpret_cast<uint64_t>(m)),
                 "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}

// 3-D tiled TMA load (no multicast) completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

// L2 policy for data read once per pass (streamed weights, K/V stages): its
// lines leave L2 first, so what the epilogues and the next kernel read
// (instructions, residual rows, partial sums, prefetched tiles) stays.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// tma_load_3d with an L2 cache policy.
__device__ __forceinline__ void tma_load_3d_hint(void* dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1, int c2,
                                                 uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, "
        "%4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "l"(pol)
        : "memory");
}

// ---- tcgen05 (5th-generation tensor core, accumulators in tensor memory)
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    __syncwarp();  // .sync.aligned: the whole warp, converged
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    __syncwarp();  // .sync.aligned: the whole warp, converged
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    __syncwarp();  // .sync.aligned: the whole warp, converged
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16, one elected thread.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every tcgen05 op issued so far by this thread is done.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 bit x 16 columns: thread i of the warp gets lane (base+i).
// The load and its wait are one asm statement: the destination registers
// hold no data until the wait has executed, and as separate statements the
// compiler may copy them in between.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    __syncwarp();  // .sync.aligned: the whole warp, converged
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor for a K-major operand laid out in 128-byte
// swizzled rows (8-row atoms of 1024 bytes).  SBO = 1024 B, LBO unused (1),
// descriptor version 1, layout SWIZZLE_128B (2).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}

// Instruction descriptor, kind::f16: fp16 A and B, fp32 accumulator, both
// operands K-major, M x N tile.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int m, int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

}  // namespace npub

// ---- thread-block clusters (2-CTA tensor-core pairs); no multicast anywhere
namespace npub {

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t nclusters_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
// CTA-wide barrier for code where lanes of a warp may arrive separately
// (role loops run by lane 0 only).  The non-.aligned form counts threads, not
// warps: __syncthreads() (bar.sync, .aligned) was measured here to release
// threads before every warp of such a CTA had arrived, even after __syncwarp().
__device__ __forceinline__ void cta_sync_divergent() { asm volatile("barrier.sync 0;" ::: "memory"); }

// Cluster-wide barrier; the non-.aligned forms, for the same reason as
// cta_sync_divergent (callers reach it from lane-0-only role loops).
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
    return r;
}
// Arrive on an mbarrier given by its shared::cluster address (own or peer CTA).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait with cluster-scope acquire (pairs with remote arrivals).
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t* bar, uint32_t parity, volatile int* abort,
                                                          uint64_t limit_ns = 2000000000ull) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((it & 255u) == 0) {
            if (*abort) return false;
            if (globaltimer_ns() - t0 > limit_ns) return false;
        }
    }
}
// Arrive on a (possibly remote) mbarrier with release semantics at cluster
// scope, and the matching acquire wait: stores a thread made (to shared::cluster
// addresses) before the arrive are visible to the threads that see the phase.
__device__ __forceinline__ void mbar_arrive_rel_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_acq_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_acq_cluster(uint64_t* bar, uint32_t parity, volatile int* abort,
                                                      uint64_t limit_ns = 2000000000ull) {
    if (mbar_try_wait_acq_cluster(bar, parity)) return true;
    uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait_acq_cluster(bar, parity)) return true;
        if ((it & 255u) == 0) {
            if (*abort) return false;
            if (globaltimer_ns() - t0 > limit_ns) return false;
        }
    }
}
// 16-byte store to another CTA's shared memory (distributed shared memory).
__device__ __forceinline__ void st_cluster_f4(uint32_t cluster_addr, const float* v) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_addr), "f"(v[0]), "f"(v[1]),
                 "f"(v[2]), "f"(v[3])
                 : "memory");
}
__device__ __forceinline__ void fence_acq_rel_cluster() { asm volatile("fence.acq_rel.cluster;" ::: "memory"); }
// The two halves of cluster_sync(), for threads that finish their remote work
// at different points: arrive when done, wait before leaving.
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }

// 3-D TMA load whose completion is signalled on a barrier that may live in the
// peer CTA of a 2-CTA pair (cta_group::2 form, no multicast).
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* m, uint32_t bar_cluster_addr, int c0,
                                                 int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
        "%5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster_addr), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
    __syncwarp();  // .sync.aligned: the whole warp, converged
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    __syncwarp();  // .sync.aligned: the whole warp, converged
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    __syncwarp();  // .sync.aligned: the whole warp, converged
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Pair MMA issued by the even CTA: D (both CTAs' TMEM) (+)= A (both CTAs' smem) * B^T.
__device__ __forceinline__ void tc_mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on the barrier at shared::cluster address `bar` (own or peer CTA) once
// the pair MMAs issued so far have completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar_cluster_addr) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster_addr)
                 : "memory");
}

}  // namespace npub

namespace npub {
// Shared-memory descriptor for an MN-major operand in 128-byte swizzled rows:
// each row holds 64 fp16 of the MN dimension for one K index; 8-row groups
// (K) are `sbo` bytes apart and 64-wide MN blocks `lbo` bytes apart.
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}
// Instruction descriptor, kind::f16, fp16 inputs, fp32 accumulator, A K-major,
// B MN-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16_bmn(int m, int n) {
    return umma_idesc_f16(m, n) | (1u << 16);
}
}  // namespace npub

namespace npub {
// 32 lanes x 32 bit x 64 columns into r[0..63], load and wait in one asm
// statement (see tmem_ld16).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
    __syncwarp();  // .sync.aligned: the whole warp, converged
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,"
        "%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
          "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
          "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
          "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr)
        : "memory");
}
// Hardware base-2 exponential (MUFU ex2, approximate, flush-to-zero).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ---- int8 weight conversion into tensor memory (W8A16 kernels)
__device__ __forceinline__ uint32_t i8_perm_lo(uint32_t u) { return __byte_perm(u, 0x64646464u, 0x5140); }
__device__ __forceinline__ uint32_t i8_perm_hi(uint32_t u) { return __byte_perm(u, 0x64646464u, 0x5342); }
__device__ __forceinline__ uint32_t f16x2_sub1152(uint32_t h) {
    __half2 v = *reinterpret_cast<__half2*>(&h);
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
    __half2 r = __hsub2(v, bias);
    return *reinterpret_cast<uint32_t*>(&r);
}
// 16 int8 -> 8 fp16 pairs (even K in the low half), exact: (q ^ 0x80) placed in
// the mantissa of 1024.0 (0x6400 | byte), minus 1152.
__device__ __forceinline__ void i8x16_to_f16x2(uint4 raw, uint32_t* o) {
    const uint32_t w0 = raw.x ^ 0x80808080u, w1 = raw.y ^ 0x80808080u, w2 = raw.z ^ 0x80808080u,
                   w3 = raw.w ^ 0x80808080u;
    o[0] = f16x2_sub1152(i8_perm_lo(w0));
    o[1] = f16x2_sub1152(i8_perm_hi(w0));
    o[2] = f16x2_sub1152(i8_perm_lo(w1));
    o[3] = f16x2_sub1152(i8_perm_hi(w1));
    o[4] = f16x2_sub1152(i8_perm_lo(w2));
    o[5] = f16x2_sub1152(i8_perm_hi(w2));
    o[6] = f16x2_sub1152(i8_perm_lo(w3));
    o[7] = f16x2_sub1152(i8_perm_hi(w3));
}

// 32 lanes x 32 columns of 32 bit from registers into tensor memory.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    __syncwarp();  // .sync.aligned: the whole warp, converged
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
        "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
        "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
        "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
    __syncwarp();
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16, A K-major in tensor memory
// (one row per lane, two fp16 per 32-bit column).
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// SwiGLU of one fp16-rounded gate / up pair (legalize.py:130-149): the one
// expression every kernel that forms it uses, so fused and separate paths
// give the same bits.  CUDA's fast exp and divide intrinsics: in a GEMM
// epilogue the full-precision forms cost more issue slots than the rest of
// the epilogue; their error (a few ulp of fp32) is far below the fp16 store.
// For g below about -88, exp overflows and the quotient is 0, as silu(g) ~ 0.
__device__ __forceinline__ float swiglu_f(float g, float u) { return __fdividef(g, 1.0f + __expf(-g)) * u; }

// The SwiGLU epilogue of a W8A16 gate|up tile with interleaved rows: lanes
// 2i and 2i + 1 hold gate and up of one channel for the same 16 tokens
// (fp16-rounded values).  The even lane forms tokens 0-7, the odd lane
// tokens 8-15; `out` gets the 8 results and *first the token offset (0 / 8).
__device__ __forceinline__ void swiglu_pair16(const float (&mine)[16], int lane, float (&out)[8], int* first) {
    const bool odd = lane & 1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float other = __shfl_xor_sync(0xffffffffu, odd ? mine[j] : mine[8 + j], 1);
        out[j] = odd ? swiglu_f(other, mine[8 + j]) : swiglu_f(mine[j], other);
    }
    *first = odd ? 8 : 0;
}
}  // namespace npub

// Execution of whole NPU programs (program_memory.bin words + a G-buffer) on
// the GPU: the drop-in for the reference's run() (b_program_examples/npu.py:62-71,
// d_compiler/npu_compiler/runtime.py:46-77), which writes the two files and
// runs the cmodel (_poc/mysim.cpp:42-157) in a subprocess.
//
// The NPU's instruction stream is straight-line (no branches), and every
// address, length and tile shape comes from the set-address / vlen / tile
// instructions before it, so the whole program is decoded on the host:
//
//  1. Decode.  The control registers are followed statically; each compute
//     instruction becomes a task reading G-buffer ranges (what its load put
//     in the PE input buffers) and writing a fresh temporary (the PE output
//     buffer, renamed per compute); each save becomes a task that rounds a
//     temporary to fp16 into a G-buffer range.  A load whose G range is
//     overwritten before its compute ran is first copied into a temporary
//     (copy task), so every task reads what the cmodel's load saw.
//  2. Schedule.  A task's level is one past the levels of the tasks it
//     depends on: earlier writers of the words it reads or writes, earlier
//     readers of the words it writes, the producers of its temporaries.
//     Tasks of one level are independent.  Freed temporaries are reused
//     (size classes), never by a task of the same or an earlier level than
//     their last reader.
//  3. Execute.  One cooperative kernel walks the levels; the CTAs share the
//     level's work in chunks and meet at a grid barrier (bounded wait) between
//     levels.  The G-buffer lives in fp32 (its values are always fp16
//     representable) at the start of one array, the temporaries after it.
//
// Arithmetic is the cmodel's (isa_semantics.cuh): float32, round-to-nearest,
// no contraction (the matmul accumulates a += x * y in ascending k with two
// roundings per step), SSE NaN results, x86-64 conversions for the
// integer-valued ops, fp16 round on save.  exp and the x^2 * sigmoid(x)
// activation use CUDA's expf (a few float32 ulps from the host libm);
// everything else gives the cmodel's bits.
#include "common.cuh"
#include "gemm_tc.h"
#include "isa_semantics.cuh"

#include <algorithm>
#include <cstring>
#include <map>
#include <new>
#include <vector>

namespace npub {
namespace prog {

enum : uint32_t { kElem = 0, kMatmul = 1, kSave = 2, kCopy = 3 };

struct Task {
    uint32_t word;  // compute instruction word (kElem / kMatmul)
    uint32_t kind;
    int32_t rA, cA, cB, pad;
    int64_t n;                    // outputs
    int64_t in1, in2, prev, out;  // offsets into the unified array; -1: none
};
static_assert(sizeof(Task) == 64, "task layout");

struct Chunk {
    int32_t task, start;
};

constexpr int kThreads = 256;
constexpr int kElemChunk = 1024;  // outputs per chunk (4 per thread)
constexpr int kMatChunk = 256;    // matmul outputs per chunk (1 per thread)

// Device view of a loaded program.
struct Dev {
    const Task* tasks;
    const Chunk* chunks;
    const int64_t* level_begin;  // [levels + 1] into chunks
    float* U;                    // [gext G words | temporaries]
    unsigned* bar;               // [0] arrivals, [1] generation, [2] abort
    int* err;
    int levels;
    uint64_t wait_ns;
};

// ---------------------------------------------------------------- device side

__device__ void run_chunk(const Dev& d, const Chunk ch) {
    const Task t = d.tasks[ch.task];
    float* U = d.U;
    if (t.kind == kMatmul) {
        const int64_t i = (int64_t)ch.start + threadIdx.x;
        if (i >= t.n) return;
        const int r = (int)(i / t.cB), c = (int)(i % t.cB);
        const float* a = U + t.in1 + (int64_t)r * t.cA;
        const float* b = U + t.in2 + c;
        float acc = 0.0f;
        for (int k = 0; k < t.cA; ++k) acc = isa::add(acc, isa::mul(a[k], b[(int64_t)k * t.cB]));
        if ((t.word >> 29) & 1u) acc = isa::act(acc, true);
        U[t.out + i] = acc;
        return;
    }
    const int64_t end = min((int64_t)ch.start + kElemChunk, t.n);
    for (int64_t i = (int64_t)ch.start + threadIdx.x; i < end; i += kThreads) {
        if (t.kind == kSave) {
            U[t.out + i] = isa::round_f16(U[t.in1 + i]);
        } else if (t.kind == kCopy) {
            U[t.out + i] = U[t.in1 + i];
        } else {
            const uint32_t op = t.word & 0xFFu;
            const int mode = (int)((t.word >> 30) & 3u);
            const float a = U[t.in1 + i];
            const float b = (t.in2 >= 0 && mode == 2) ? U[t.in2 + i] : (float)((t.word >> 8) & 0xFFFFu);
            const float p = (op == 0x0Cu && t.prev >= 0) ? U[t.prev + i] : 0.0f;
            U[t.out + i] = isa::elem_op(t.word, a, b, p);
        }
    }
}

// Grid barrier for a cooperative launch: arrivals counted in bar[0], the
// last arrival bumps the generation bar[1].  The wait is bounded: on time-out
// the CTA raises bar[2] and the error word, and every CTA leaves at its next
// barrier.  Returns false when the run is being abandoned.
__device__ bool grid_barrier(const Dev& d) {
    __syncthreads();
    __shared__ int ok_s;
    if (threadIdx.x == 0) {
        volatile unsigned* gen = d.bar + 1;
        const unsigned g0 = *gen;
        __threadfence();
        const unsigned arrived = atomicAdd(d.bar, 1u);
        bool ok = true;
        if (arrived == gridDim.x - 1) {
            d.bar[0] = 0u;
            __threadfence();
            atomicAdd(d.bar + 1, 1u);
        } else {
            const uint64_t t0 = globaltimer_ns();
            for (uint32_t it = 1; *gen == g0; ++it) {
                if ((it & 255u) == 0 && (*(volatile unsigned*)(d.bar + 2) || globaltimer_ns() - t0 > d.wait_ns)) {
                    ok = false;
                    break;
                }
            }
        }
        __threadfence();
        if (!ok) {
            atomicExch(d.bar + 2, 1u);
            if (d.err) atomicCAS(d.err, 0, 0x601);
        }
        ok_s = ok && !*(volatile unsigned*)(d.bar + 2);
    }
    __syncthreads();
    return ok_s != 0;
}

__global__ void __launch_bounds__(kThreads) program_kernel(const Dev d) {
    for (int L = 0; L < d.levels; ++L) {
        const int64_t c0 = d.level_begin[L], c1 = d.level_begin[L + 1];
        for (int64_t c = c0 + blockIdx.x; c < c1; c += gridDim.x) run_chunk(d, d.chunks[c]);
        if (gridDim.x == 1) {
            __syncthreads();
        } else if (!grid_barrier(d)) {
            return;
        }
    }
}

// G words of the unified array -> fp16 words (beyond gext: +0, as the cmodel's write-back).
__global__ void gbuf_out_kernel(const float* U, int64_t gext, uint16_t* out, int64_t gn) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < gn; i += (int64_t)gridDim.x * blockDim.x) {
        out[i] = isa::f16_bits(i < gext ? U[i] : 0.0f);
    }
}

// fp16 input words -> the G region (beyond n_in: zeros, the cmodel's fresh buffer).
__global__ void gbuf_in_kernel(const uint16_t* in, int64_t n_in, float* U, int64_t gext) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < gext; i += (int64_t)gridDim.x * blockDim.x)
        U[i] = i < n_in ? isa::h2f(in[i]) : 0.0f;
}

// ---------------------------------------------------------------- host side

struct Program {
    std::vector<Task> tasks;
    std::vector<Chunk> chunks;
    std::vector<int64_t> level_begin;
    int64_t gext = 0;      // G words the machine holds (input, growth, default capacity)
    int64_t tsize = 0;     // temporaries (floats)
    int64_t executed = 0;  // program-counter steps taken
    int grid = 1;
    // workspace layout (bytes)
    size_t off_tasks = 0, off_chunks = 0, off_levels = 0, off_bar = 0, off_U = 0, total = 0;
};

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Level bookkeeping of the G-buffer words and of the temporaries.
struct Scheduler {
    std::vector<int32_t> lastW, lastR;  // per G word
    void grow(int64_t n) {
        if ((int64_t)lastW.size() < n) {
            lastW.resize(n, 0);
            lastR.resize(n, 0);
        }
    }
    int32_t read_dep(int64_t b, int64_t n) const {
        int32_t m = 0;
        for (int64_t i = b; i < b + n; ++i) m = std::max(m, lastW[i]);
        return m;
    }
    int32_t write_dep(int64_t b, int64_t n) const {
        int32_t m = 0;
        for (int64_t i = b; i < b + n; ++i) m = std::max(m, std::max(lastW[i], lastR[i]));
        return m;
    }
    void mark_read(int64_t b, int64_t n, int32_t L) {
        for (int64_t i = b; i < b + n; ++i) lastR[i] = std::max(lastR[i], L);
    }
    void mark_write(int64_t b, int64_t n, int32_t L) {
        for (int64_t i = b; i < b + n; ++i) lastW[i] = L;
    }
};

// A temporary: a range of the temp region with the level of the task that
// wrote it and the highest level that read it.
struct Temp {
    int64_t off = -1, size = 0;
    int32_t wlevel = 0, rlevel = 0;
    bool live = false;
};

struct TempPool {
    std::vector<Temp> all;
    std::map<int, std::vector<int>> free_by_class;  // size class -> temp ids
    int64_t top = 0;
    static int size_class(int64_t n) {
        int c = 6;
        while ((int64_t(1) << c) < n) ++c;
        return c;
    }
    // A temporary of >= n floats that a task at level L0 may overwrite (its
    // previous value was written and read at lower levels), or a new one.
    int take(int64_t n, int32_t& L0) {
        const int c = size_class(n);
        auto& fl = free_by_class[c];
        for (size_t k = 0; k < fl.size(); ++k) {
            Temp& t = all[fl[k]];
            if (std::max(t.wlevel, t.rlevel) < L0) {
                const int id = fl[k];
                fl[k] = fl.back();
                fl.pop_back();
                t.live = true;
                return id;
            }
        }
        Temp t;
        t.size = int64_t(1) << c;
        t.off = top;
        top += t.size;
        t.live = true;
        all.push_back(t);
        return (int)all.size() - 1;
    }
    void release(int id) {
        if (id < 0 || !all[id].live) return;
        all[id].live = false;
        free_by_class[size_class(all[id].size)].push_back(id);
    }
};

// What a PE input buffer holds: a G range as of its load, or a temporary.
struct PeIn {
    bool valid = false;
    int64_t gbase = 0, n = 0;
    int temp = -1;  // materialised copy
};

// Program counter of the instruction a failed decode stopped at (this thread).
static thread_local int t_error_pc = -1;

struct Decoded {
    std::vector<Task> tasks;
    std::vector<int32_t> level;     // per task
    std::vector<int32_t> temp_out;  // per task: the temp it writes (-1 for saves)
};

static int decode(const uint32_t* words, int64_t nwords, int64_t maxrun, int64_t g_in, Program& P) {
    uint32_t blo[3] = {0, 0, 0}, bhi[3] = {0, 0, 0};
    int64_t vlen = 0, tA[2] = {0, 0}, tB[2] = {0, 0};
    Scheduler S;
    TempPool pool;
    PeIn pe[2];
    int out_temp = -1;     // the PE output buffer (renamed)
    int64_t out_n = 0;
    Decoded D;
    // the cmodel's G-buffer starts at max(65536, input) words and grows on demand
    int64_t gext = std::max<int64_t>(65536, g_in);
    S.grow(gext);
    auto base = [&](int o) { return (int64_t)(blo[o] | ((uint64_t)bhi[o] << 16)); };
    auto need_g = [&](int64_t end) {
        if (end > gext) {
            gext = end;
            S.grow(gext);
        }
    };
    auto add_task = [&](const Task& t, int32_t L, int tout) {
        D.tasks.push_back(t);
        D.level.push_back(L);
        D.temp_out.push_back(tout);
    };
    // a G-range input of a task at level L, or the temp it was copied to
    auto in_dep = [&](const PeIn& p, int64_t n) -> int32_t {
        if (p.temp >= 0) return pool.all[p.temp].wlevel;
        return S.read_dep(p.gbase, n);
    };
    auto in_mark = [&](const PeIn& p, int64_t n, int32_t L) {
        if (p.temp >= 0) {
            Temp& t = pool.all[p.temp];
            t.rlevel = std::max(t.rlevel, L);
        } else {
            S.mark_read(p.gbase, n, L);
        }
    };
    auto in_off = [&](const PeIn& p) -> int64_t { return p.temp >= 0 ? -2 - p.temp : p.gbase; };  // temp: fixed later

    int64_t pc = 0;
    const int64_t steps = maxrun;
    for (pc = 0; pc < steps; ++pc) {
        const uint32_t w = pc < nwords ? words[pc] : 0u;
        const uint32_t op = w & 0xFFu;
        const int mode = (int)((w >> 30) & 3u);
        if (op == 0xFFu) {
            ++pc;
            break;
        }
        if (w == 0) continue;
        if (op == 0x80u) {
            const int o = (int)((w >> 30) & 3u);
            const uint32_t v = (w >> 8) & 0xFFFFu;
            if (o < 3) {
                if ((w >> 29) & 1u) bhi[o] = v; else blo[o] = v;
            }
        } else if (op == 0x82u) {
            vlen = (int64_t)((w >> 8) & 0xFFFFu);
        } else if (op == 0x88u) {
            const int m = (int)((w >> 31) & 1u);
            tA[m] = (int64_t)((w >> 8) & 0xFFu);
            tB[m] = (int64_t)((w >> 16) & 0xFFu);
        } else if (op == 0x90u) {
            const int matrix = (int)((w >> 31) & 1u), o = (int)((w >> 30) & 1u);
            const int64_t b = base(o), n = matrix ? tA[o] * tB[o] : vlen;
            need_g(b + n);
            if (pe[o].temp >= 0) pool.release(pe[o].temp);
            pe[o] = PeIn();
            pe[o].valid = true;
            pe[o].gbase = b;
            pe[o].n = n;
        } else if (op == 0x98u) {
            const int64_t b = base(2), n = out_n;
            if (n == 0) continue;
            need_g(b + n);
            // loads whose G range this save overwrites keep what they read: copy them first
            for (int s = 0; s < 2; ++s) {
                PeIn& p = pe[s];
                if (!p.valid || p.temp >= 0 || p.n == 0 || p.gbase >= b + n || b >= p.gbase + p.n) continue;
                int32_t L = 1 + S.read_dep(p.gbase, p.n);
                const int t = pool.take(p.n, L);
                Task c{};
                c.kind = kCopy;
                c.n = p.n;
                c.in1 = p.gbase;
                c.in2 = c.prev = -1;
                c.out = -2 - t;
                S.mark_read(p.gbase, p.n, L);
                pool.all[t].wlevel = L;
                pool.all[t].rlevel = 0;
                add_task(c, L, t);
                p.temp = t;
            }
            Temp& src = pool.all[out_temp];
            const int32_t L = 1 + std::max(src.wlevel, S.write_dep(b, n));
            Task t{};
            t.kind = kSave;
            t.n = n;
            t.in1 = -2 - out_temp;
            t.in2 = t.prev = -1;
            t.out = b;
            src.rlevel = std::max(src.rlevel, L);
            S.mark_write(b, n, L);
            add_task(t, L, -1);
        } else {
            const bool matrix = op >= 0x40u && op <= 0x43u;
            const bool is_mm = matrix && op == 0x42u && mode == 2;
            Task t{};
            t.word = w;
            t.in2 = t.prev = -1;
            int32_t L = 0;
            int64_t n;
            if (is_mm) {
                const int64_t rA = tA[0], cA = tB[0], cB = tB[1];
                n = rA * cB;
                // an input never loaded is an empty PE buffer (the cmodel's empty vector)
                if ((rA * cA > 0 && (!pe[0].valid || pe[0].n < rA * cA)) ||
                    (cA * cB > 0 && (!pe[1].valid || pe[1].n < cA * cB))) {
                    t_error_pc = (int)pc;
                    return NPUB_ERR_INVALID_ARG;  // the cmodel would read past a PE buffer
                }
                t.kind = kMatmul;
                t.rA = (int32_t)rA;
                t.cA = (int32_t)cA;
                t.cB = (int32_t)cB;
                t.n = n;
                L = std::max(in_dep(pe[0], rA * cA), in_dep(pe[1], cA * cB));
                t.in1 = in_off(pe[0]);
                t.in2 = in_off(pe[1]);
            } else {
                n = matrix ? tA[0] * tB[0] : vlen;
                // the ops whose result reads the second operand (mysim.cpp:117-136)
                const bool reads_b = op == 0x01u || op == 0x02u || op == 0x08u || op == 0x09u || op == 0x0Au ||
                                     op == 0x0Bu || op == 0x0Cu || op == 0x0Du || op == 0x11u || op == 0x12u ||
                                     (op >= 0x40u && op <= 0x43u);
                const bool uses_in2 = reads_b && mode == 2;
                if (!pe[0].valid || pe[0].n < n || (uses_in2 && (!pe[1].valid || pe[1].n < n))) {
                    if (n > 0) {
                        t_error_pc = (int)pc;
                        return NPUB_ERR_INVALID_ARG;
                    }
                }
                t.kind = kElem;
                t.n = n;
                if (n > 0) {
                    L = in_dep(pe[0], n);
                    t.in1 = in_off(pe[0]);
                    if (uses_in2) {
                        L = std::max(L, in_dep(pe[1], n));
                        t.in2 = in_off(pe[1]);
                    }
                }
                // mul-add reads the previous PE output when it has this size (else zeros)
                if (op == 0x0Cu && out_temp >= 0 && out_n == n && n > 0) {
                    L = std::max(L, pool.all[out_temp].wlevel);
                    t.prev = -2 - out_temp;
                }
            }
            L += 1;
            const int old_out = out_temp;
            int tout = -1;
            if (n > 0) {
                int32_t L2 = L;
                tout = pool.take(n, L2);
                L = std::max(L, L2);
                t.out = -2 - tout;
                if (is_mm) {
                    in_mark(pe[0], t.rA * (int64_t)t.cA, L);
                    in_mark(pe[1], t.cA * (int64_t)t.cB, L);
                } else {
                    in_mark(pe[0], n, L);
                    if (t.in2 != -1) in_mark(pe[1], n, L);
                    if (t.prev != -1) pool.all[old_out].rlevel = std::max(pool.all[old_out].rlevel, L);
                }
                pool.all[tout].wlevel = L;
                pool.all[tout].rlevel = 0;
                add_task(t, L, tout);
            }
            if (old_out >= 0) pool.release(old_out);
            out_temp = tout;
            out_n = n;
        }
    }
    P.executed = pc;
    P.gext = gext;
    P.tsize = pool.top;
    // resolve temp offsets (after the G region) and lay the tasks out by level
    const int64_t T = (int64_t)D.tasks.size();
    auto fix = [&](int64_t v) { return v <= -2 ? gext + pool.all[-2 - v].off : v; };
    int32_t levels = 0;
    for (int64_t i = 0; i < T; ++i) levels = std::max(levels, D.level[i]);
    {  // levels without tasks need no barrier: renumber the used ones 1..K
        std::vector<int32_t> rank(levels + 1, 0);
        for (int64_t i = 0; i < T; ++i) rank[D.level[i]] = 1;
        int32_t k = 0;
        for (int32_t l = 1; l <= levels; ++l)
            if (rank[l]) rank[l] = ++k;
        for (int64_t i = 0; i < T; ++i) D.level[i] = rank[D.level[i]];
        levels = k;
    }
    std::vector<int64_t> cnt(levels + 2, 0);
    for (int64_t i = 0; i < T; ++i) cnt[D.level[i]]++;
    std::vector<int64_t> pos(levels + 2, 0);
    for (int32_t l = 1; l <= levels; ++l) pos[l + 1] = pos[l] + cnt[l];
    P.tasks.assign(T, Task{});
    std::vector<int64_t> order(T);
    for (int64_t i = 0; i < T; ++i) {
        Task t = D.tasks[i];
        t.in1 = fix(t.in1);
        t.in2 = fix(t.in2);
        t.prev = fix(t.prev);
        t.out = fix(t.out);
        const int64_t k = pos[D.level[i]]++;
        P.tasks[k] = t;
        order[k] = D.level[i];
    }
    P.level_begin.assign(levels + 1, 0);
    P.chunks.clear();
    int64_t max_chunks = 1;
    int64_t k = 0;
    for (int32_t l = 1; l <= levels; ++l) {
        P.level_begin[l - 1] = (int64_t)P.chunks.size();
        for (; k < T && order[k] == l; ++k) {
            const Task& t = P.tasks[k];
            const int step = t.kind == kMatmul ? kMatChunk : kElemChunk;
            for (int64_t s = 0; s < t.n; s += step) P.chunks.push_back(Chunk{(int32_t)k, (int32_t)s});
        }
        max_chunks = std::max<int64_t>(max_chunks, (int64_t)P.chunks.size() - P.level_begin[l - 1]);
    }
    P.level_begin[levels] = (int64_t)P.chunks.size();
    P.grid = (int)std::min<int64_t>(max_chunks, (int64_t)num_sms());
    if (P.grid < 1) P.grid = 1;
    P.off_tasks = 0;
    P.off_chunks = align256(P.off_tasks + P.tasks.size() * sizeof(Task));
    P.off_levels = align256(P.off_chunks + P.chunks.size() * sizeof(Chunk));
    P.off_bar = align256(P.off_levels + P.level_begin.size() * sizeof(int64_t));
    P.off_U = align256(P.off_bar + 4 * sizeof(unsigned));
    P.total = align256(P.off_U + (size_t)(P.gext + P.tsize) * sizeof(float));
    return NPUB_OK;
}

}  // namespace prog
}  // namespace npub

using namespace npub;

extern "C" int npub_program_create(const uint32_t* words, int64_t nwords, int64_t maxrun, int64_t g_in,
                                   void** program) {
    NPUB_CHECK_ARG(program && nwords >= 0 && maxrun >= 0 && g_in >= 0);
    NPUB_CHECK_ARG(words || nwords == 0);
    *program = nullptr;
    prog::t_error_pc = -1;
    prog::Program* P = new (std::nothrow) prog::Program();
    if (!P) return NPUB_ERR_UNSUPPORTED;
    int rc;
    try {
        rc = prog::decode(words, nwords, maxrun, g_in, *P);
    } catch (const std::bad_alloc&) {
        rc = NPUB_ERR_UNSUPPORTED;
    }
    if (rc != NPUB_OK) {
        delete P;
        return rc;
    }
    *program = P;
    return NPUB_OK;
}

extern "C" int npub_program_info(const void* program, int64_t* info, int n) {
    NPUB_CHECK_ARG(program && info && n >= 0);
    const prog::Program* P = reinterpret_cast<const prog::Program*>(program);
    const int64_t v[7] = {P->executed, (int64_t)P->tasks.size(), (int64_t)P->level_begin.size() - 1, P->gext,
                          P->tsize, (int64_t)P->chunks.size(), P->grid};
    for (int i = 0; i < n && i < 7; ++i) info[i] = v[i];
    return NPUB_OK;
}

extern "C" size_t npub_program_workspace(const void* program) {
    return program ? reinterpret_cast<const prog::Program*>(program)->total : 0;
}

extern "C" int npub_program_load(const void* program, void* workspace, size_t workspace_bytes, void* stream) {
    NPUB_CHECK_ARG(program && workspace);
    const prog::Program* P = reinterpret_cast<const prog::Program*>(program);
    if (workspace_bytes < P->total) return NPUB_ERR_WORKSPACE;
    NPUB_CHECK_ARG(npub_aligned(workspace, 256));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    if (!P->tasks.empty())
        NPUB_CUDA_TRY(cudaMemcpyAsync(ws + P->off_tasks, P->tasks.data(), P->tasks.size() * sizeof(prog::Task),
                                      cudaMemcpyHostToDevice, st));
    if (!P->chunks.empty())
        NPUB_CUDA_TRY(cudaMemcpyAsync(ws + P->off_chunks, P->chunks.data(), P->chunks.size() * sizeof(prog::Chunk),
                                      cudaMemcpyHostToDevice, st));
    NPUB_CUDA_TRY(cudaMemcpyAsync(ws + P->off_levels, P->level_begin.data(), P->level_begin.size() * sizeof(int64_t),
                                  cudaMemcpyHostToDevice, st));
    // the tables are read from the host copy while the copies are queued
    NPUB_CUDA_TRY(cudaStreamSynchronize(st));
    return NPUB_OK;
}

extern "C" int npub_program_run(const void* program, const uint16_t* g_in, int64_t n_in, uint16_t* g_out, int64_t gn,
                                void* workspace, size_t workspace_bytes, void* stream) {
    NPUB_CHECK_ARG(program && workspace && n_in >= 0 && gn >= 0);
    NPUB_CHECK_ARG(g_in || n_in == 0);
    NPUB_CHECK_ARG(g_out || gn == 0);
    const prog::Program* P = reinterpret_cast<const prog::Program*>(program);
    if (workspace_bytes < P->total) return NPUB_ERR_WORKSPACE;
    NPUB_CHECK_ARG(npub_aligned(workspace, 256));
    NPUB_CHECK_ARG(n_in <= P->gext);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    prog::Dev d;
    d.tasks = reinterpret_cast<const prog::Task*>(ws + P->off_tasks);
    d.chunks = reinterpret_cast<const prog::Chunk*>(ws + P->off_chunks);
    d.level_begin = reinterpret_cast<const int64_t*>(ws + P->off_levels);
    d.U = reinterpret_cast<float*>(ws + P->off_U);
    d.bar = reinterpret_cast<unsigned*>(ws + P->off_bar);
    d.err = npub_internal_device_error_word();
    d.levels = (int)P->level_begin.size() - 1;
    d.wait_ns = npub_internal_wait_limit_ns();
    NPUB_CUDA_TRY(cudaMemsetAsync(d.bar, 0, 4 * sizeof(unsigned), st));
    const int gb = (int)std::min<int64_t>((P->gext + 255) / 256, (int64_t)num_sms() * 8);
    prog::gbuf_in_kernel<<<gb > 0 ? gb : 1, 256, 0, st>>>(g_in, n_in, d.U, P->gext);
    int rc = npub_internal_launch_status();
    if (rc) return rc;
    if (d.levels > 0) {
        void* args[] = {&d};
        const cudaError_t e = cudaLaunchCooperativeKernel((void*)prog::program_kernel, dim3(P->grid),
                                                          dim3(prog::kThreads), args, 0, st);
        if (e != cudaSuccess) {
            npub_internal_set_cuda_error(e);
            return NPUB_ERR_CUDA;
        }
        rc = npub_internal_launch_status();
        if (rc) return rc;
    }
    if (gn > 0) {
        const int ob = (int)std::min<int64_t>((gn + 255) / 256, (int64_t)num_sms() * 8);
        prog::gbuf_out_kernel<<<ob, 256, 0, st>>>(d.U, P->gext, g_out, gn);
        return npub_internal_launch_status();
    }
    return NPUB_OK;
}

extern "C" int npub_program_error_pc(void) { return prog::t_error_pc; }

extern "C" int npub_program_destroy(void* program) {
    delete reinterpret_cast<prog::Program*>(program);
    return NPUB_OK;
}

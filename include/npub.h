/*
 * npub.h -- C ABI of libnpub, the sm_100a (B200) implementation of the compute
 * that KwanyoungCho/NPU_COMP lowers onto its NPU: the W8A16 matmul and the
 * Llama-layer vector ops (RMSNorm, SwiGLU, softmax/exp, RoPE, attention),
 * plus the NPU's elementwise instruction semantics.
 *
 * Conventions
 *   - Every pointer argument named as a tensor is a DEVICE pointer owned by
 *     the caller.  fp16 tensors are passed as `void*` (IEEE binary16), int8
 *     weights as `int8_t*`, fp32 buffers as `float*`.
 *   - Leading dimensions (`ld*`) are in elements.  Matrices are row-major.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Every call is
 *     stream-ordered and asynchronous; nothing allocates device memory.
 *     Calls that need scratch take a caller-provided workspace and report its
 *     size through the matching *_workspace() query.
 *   - Every call returns an int status: NPUB_OK (0) or a negative NPUB_ERR_*.
 *     No C++ exception crosses this boundary.  npub_strerror() names a status.
 *   - Entry points are thread-safe; the per-device state (driver entry point,
 *     SM count, device error word) is created once under a lock.
 *
 * Reference interface replaced (paths inside KwanyoungCho/NPU_COMP):
 *   b_program_examples/npu.py:41-47   matmul(asm, aAddr, bAddr, cAddr, M, K, N, act)
 *   b_program_examples/npu.py:62-71   run(asm, gbuf, gn, rundir, maxrun)
 *   _poc/mysim.cpp:83-145             the cmodel's execute loop that run() drives
 *   b_program_examples/llama_layer.py:71-152   vec/unary/rmsnorm/rope/attention/FFN macros
 *   d_compiler/npu_compiler/legalize.py:20-149 the compiler's op recipes
 */
#ifndef NPUB_H
#define NPUB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  Failures of the reference's CPU path surface as a
 * CalledProcessError from subprocess.run(check=True) (npu.py:66-69) or a
 * CodegenError (d_compiler/npu_compiler/codegen.py:21-22); here they are
 * return codes. */
#define NPUB_OK 0
#define NPUB_ERR_INVALID_ARG (-1)    /* bad shape, stride, alignment or null pointer */
#define NPUB_ERR_UNSUPPORTED (-2)    /* valid request outside what the kernels implement */
#define NPUB_ERR_CUDA (-3)           /* a CUDA runtime/driver call failed (see npub_last_cuda_error) */
#define NPUB_ERR_WORKSPACE (-4)      /* workspace missing or smaller than *_workspace() */
#define NPUB_ERR_DEVICE_TIMEOUT (-5) /* a bounded device-side wait gave up (npub_device_error) */
#define NPUB_ERR_NO_DEVICE (-6)      /* no sm_100 device current */
#define NPUB_ERR_SCRATCH_LIMIT (-7)  /* request needs more than the static scratch of npub_w8a16_gemm_noalloc */

/* Library version (major*10000 + minor*100 + patch). */
int npub_version(void);
/* Text for a status code (static storage). */
const char* npub_strerror(int status);
/* The cudaError_t of the last NPUB_ERR_CUDA on this thread (0 if none). */
int npub_last_cuda_error(void);
/* Number of kernels libnpub has launched in this process (all devices). */
unsigned long long npub_launch_count(void);
/* Reads (and with clear != 0 resets) the current device's error word, which
 * kernels set when a bounded wait gives up.  Synchronises the device.
 * Returns 0 when no kernel reported an error. */
int npub_device_error(int clear);

/* ------------------------------------------------------------------ GEMM --
 * W8A16 matmul (replaces the matmul macro b_program_examples/npu.py:41-47
 * executed by m_mul, _poc/mysim.cpp:109-113, with the weights int8 and a
 * per-output-channel scale):
 *
 *   C[m, n] = fp16( alpha * scale[n] * sum_k A[m, k] * Wq[n, k] )  (+ R[m, n])
 *
 * A    fp16 [M, K] (lda >= K, lda % 8 == 0, 16-byte aligned)
 * Wq   int8 [N, K] K-major (ldw >= K, ldw % 16 == 0, 16-byte aligned)
 * scale fp16 [N] (NULL = 1)
 * C    fp16 [M, N] (ldc >= N);  R fp16 [M, N] residual added after scaling (NULL = none)
 * K % 16 == 0.  Accumulation is fp32 on the tensor cores (tcgen05).
 * workspace: npub_w8a16_gemm_workspace(M, N, K) bytes (split-K partials);
 * may be NULL when that query returns 0.  A non-empty workspace starts with
 * 64 KiB of tile counters (used by the stream-K kernel that decode-sized M
 * runs on): they must be zero before the first call on that workspace, every
 * completed call leaves them zero again, and nothing else may write them
 * (other data, calls running at the same time on other streams).  Re-zero
 * them after a call that reported NPUB_ERR_DEVICE_TIMEOUT. */
int npub_w8a16_gemm(const void* A, int64_t lda, const int8_t* Wq, int64_t ldw, const void* scale, void* C,
                    int64_t ldc, const void* R, int64_t ldr, int M, int N, int K, float alpha, void* workspace,
                    size_t workspace_bytes, void* stream);
size_t npub_w8a16_gemm_workspace(int M, int N, int K);
/* Gate|up projection fused with SwiGLU (llama_layer.py:143-150: silu(x Wg) *
 * (x Wu), legalize.py:130-149).  Wq [2F, K] int8 holds the gate and up rows
 * interleaved -- row 2c is gate channel c, row 2c + 1 up channel c, and
 * scale [2F] likewise -- and C [M, F] (row stride ldc) receives
 * fp16(silu(g) * u) with g, u the fp16-rounded projections: the bits of
 * npub_w8a16_gemm into an [M, 2F] buffer followed by npub_swiglu on its even
 * and odd columns, without the [M, 2F] round trip through memory.  Workspace
 * as npub_w8a16_gemm for (M, 2F, K). */
int npub_w8a16_gemm_swiglu(const void* A, int64_t lda, const int8_t* Wq, int64_t ldw, const void* scale, void* C,
                           int64_t ldc, int M, int F, int K, void* workspace, size_t workspace_bytes, void* stream);
/* W8A16 GEMM of a decode step (M <= 64, the stream-K kernel) with an RMSNorm
 * folded in, replacing the RMSNorm -> projection pairs of llama_layer.py:79-89
 * -> 95-113 and :139-141 -> 143-150 (legalize.py:30-47 for the norm):
 *   consumer (rs_part != NULL): A = fp16(h * gamma) for a residual stream h and
 *     row t of the result is scaled by 1 / sqrt(sum_{i<rs_n} rs_part[i*rs_ld + t] / rs_d + rs_eps)
 *     before rounding (and before SwiGLU when swiglu != 0; C is then [M, N/2]);
 *   producer (G, ss != NULL): C = fp16(A Wq^T * scale + R) as npub_w8a16_gemm,
 *     plus G = fp16(C * gamma) [M, N] and ss[(n/32)*ss_ld + t] = sum of C[t, n]^2
 *     over the 32 columns n/32 -- the rs_part (rs_n = N / 32) of the next call.
 * npub_rmsnorm_parts() makes G and ss for a stream that no GEMM produced.
 * Wq_next (may be NULL): the next GEMM of a decode chain (same M, int8
 * [N_next, K_next], row stride ldw_next), whose first weight tiles this call
 * prefetches to L2 while its own MMAs run.
 * Returns NPUB_ERR_UNSUPPORTED for M > 64.  Workspace:
 * npub_w8a16_gemm_rms_workspace(M, N, K) bytes whose first 64 KiB are zero
 * before the first call (every call leaves them zero). */
int npub_w8a16_gemm_rms(const void* A, int64_t lda, const int8_t* Wq, int64_t ldw, const void* scale, void* C,
                        int64_t ldc, const void* R, int64_t ldr, int M, int N, int K, int swiglu,
                        const float* rs_part, int rs_n, int64_t rs_ld, int rs_d, float rs_eps, const void* gamma,
                        void* G, int64_t ldg, float* ss, int64_t ss_ld, const int8_t* Wq_next, int64_t ldw_next,
                        int N_next, int K_next, void* workspace, size_t workspace_bytes, void* stream);
size_t npub_w8a16_gemm_rms_workspace(int M, int N, int K);

/* Name of the kernel npub_w8a16_gemm runs for this shape (static storage):
 * the 2-CTA pair kernel, or the stream-K kernel for decode-sized M.  No
 * reference counterpart (diagnostics). */
const char* npub_w8a16_kernel_name(int M, int N, int K);

/* Allocation-free W8A16 matmul (no counterpart in the reference, which has no
 * device memory at all).  Same contract and result as npub_w8a16_gemm, for
 * callers that cannot allocate device memory -- a plugin whose host runtime
 * owns all device memory, a plain C/ctypes caller with no device allocator,
 * or a fixed-budget decode loop where cudaMalloc is not allowed -- and so
 * cannot pass a workspace.  The split-K scratch comes from a static device
 * array of NPUB_NOALLOC_SCRATCH_BYTES that every device loading the library
 * holds until exit.  Requests whose npub_w8a16_gemm_workspace(M, N, K)
 * exceeds that return NPUB_ERR_SCRATCH_LIMIT.  The first call on a device
 * looks up the array's device address (cudaGetSymbolAddress) with that
 * device current; make that first call before any stream capture.  All calls
 * share the array: calls that overlap on the GPU race.  Nothing is allocated. */
#define NPUB_NOALLOC_SCRATCH_BYTES (16u << 20)
int npub_w8a16_gemm_noalloc(const void* A, int64_t lda, const int8_t* Wq, int64_t ldw, const void* scale, void* C,
                            int64_t ldc, const void* R, int64_t ldr, int M, int N, int K, float alpha, void* stream);

/* Same contract with fp16 weights W [N, K] (ldw % 8 == 0): the plain fp16
 * matmul of npu.py:41-47 / mysim.cpp:109-113 on tensor cores (used for the
 * fp16 lm_head and for matmuls whose weights are not quantised). */
int npub_f16_gemm(const void* A, int64_t lda, const void* W, int64_t ldw, const void* scale, void* C, int64_t ldc,
                  const void* R, int64_t ldr, int M, int N, int K, float alpha, void* workspace,
                  size_t workspace_bytes, void* stream);
size_t npub_f16_gemm_workspace(int M, int N, int K);

/* Quantise fp32 weights W [K, N] (row-major, x @ W convention of
 * llama_layer.py:27-31) to int8 Wq [N, K] K-major with fp16 per-output-channel
 * scales:  s[n] = fp16(max_k |W[k,n]| / 127),  Wq[n,k] = clip(rint(W[k,n] / s[n]), -127, 127);
 * a column of zeros gets s = 0 and Wq = 0.  (The reference has no quantiser;
 * this is the symmetric per-channel scheme its W8A16 target is defined by.) */
int npub_quantize_w8(const float* W, int64_t ldw, int K, int N, int8_t* Wq, int64_t ldq, void* scale, void* stream);

/* ---------------------------------------------------------- vector ops --
 * RMSNorm, d_compiler/npu_compiler/legalize.py:30-47, b_program_examples/llama_layer.py:79-89:
 *   y[r, :] = fp16( x[r, :] / sqrt(mean(x[r, :]^2) + eps) * gamma )   (fp32 math)
 * x, y fp16 [rows, d] (ld % 8 == 0), gamma fp16 [d]; d % 8 == 0.
 * If `residual` is not NULL, x + residual is normalised and also written back
 * to `x_out` (fp16, may alias x) -- the residual add of llama_layer.py:139. */
int npub_rmsnorm(const void* x, int64_t ldx, const void* residual, int64_t ldr, void* x_out, int64_t ldxo,
                 const void* gamma, void* y, int64_t ldy, int rows, int d, float eps, void* stream);

/* The inputs npub_w8a16_gemm_rms takes for an RMSNorm of x (fp16 [rows, d],
 * d % 32 == 0): G = fp16(x * gamma) and ss[c*ss_ld + r] = sum_{j<32} x[r, 32c + j]^2. */
int npub_rmsnorm_parts(const void* x, int64_t ldx, const void* gamma, void* G, int64_t ldg, float* ss,
                       int64_t ss_ld, int rows, int d, void* stream);

/* Residual add, the v_add of b_program_examples/llama_layer.py:139,152:
 *   out = fp16(a + b)  (fp32 add), a, b, out fp16 [rows, cols] (out may alias a or b). */
int npub_add(const void* a, int64_t lda, const void* b, int64_t ldb, void* out, int64_t ldo, int rows, int cols,
             void* stream);

/* SwiGLU, legalize.py:130-149, llama_layer.py:143-151:
 *   h = fp16( g / (1 + exp(-g)) * u )   (fp32 math with CUDA's fast exp and
 *   divide, a few fp32 ulps; the same expression as the SwiGLU epilogue of
 *   npub_w8a16_gemm_swiglu), g, u, h fp16 [rows, cols]. */
int npub_swiglu(const void* g, int64_t ldg, const void* u, int64_t ldu, void* h, int64_t ldh, int rows, int cols,
                void* stream);

/* Row softmax, legalize.py:97-114 (mask -30000), stable form of
 * d_compiler/npu_compiler/model.py:149-150:
 *   p[b, r, c] = exp(scale*s - max) / sum(...) over c <= r + causal_offset
 * (all c when causal_offset < 0 is NPUB_NO_CAUSAL); masked entries are written
 * as 0 up to the next multiple of 128 past the diagonal (what the causal
 * context GEMM reads) or to the row end when zero_full != 0.
 * s, p fp16 [batch, rows, ld] (may alias). */
#define NPUB_NO_CAUSAL (-1)
int npub_softmax_rows(const void* s, void* p, int64_t ld, int64_t batch_stride, int batch, int rows, int cols,
                      float scale, int causal_offset, int zero_full, void* stream);

/* RoPE (rotate_half convention), llama_layer.py:33-40,96-112, legalize.py:67-94:
 *   x'[d] = x[d]*cos(p*th_i) + rh[d]*sin(p*th_i),  th_i = theta^(-2i/hd), i = d mod hd/2,
 *   rh = [-x[hd/2:], x[:hd/2]],  p = pos0 + t  (or positions[t] when not NULL).
 * In place on x fp16 [tokens, heads*head_dim] with row stride ldx; head_dim even, % 8 == 0. */
int npub_rope(void* x, int64_t ldx, int tokens, int heads, int head_dim, const int32_t* positions, int pos0,
              float theta, void* stream);

/* Token embedding and greedy selection around the layer stack (no counterpart
 * in the reference, whose programs start from hidden states):
 * npub_embed: out[r, :] = table[ids[r], :] (fp16, d % 8 == 0); ids outside
 * [0, vocab) give zeros.  npub_argmax_rows: per row the largest logit
 * (val, may be NULL) and its smallest index (idx). */
int npub_embed(const int32_t* ids, int n, const void* table, int64_t ldt, int vocab, int d, void* out, int64_t ldo,
               void* stream);
int npub_argmax_rows(const void* x, int64_t ldx, int rows, int cols, int32_t* idx, float* val, void* stream);
/* Greedy selection over a vocabulary split across tensor-parallel ranks, in
 * one exchange: npub_argmax_keys packs each row's (largest logit, its smallest
 * index + index_offset) into one uint64 key that orders by value, then by
 * smaller index; after an all-gather of the ranks' keys [ranks, rows],
 * npub_select_keys writes the winning global index of every row to ids.
 * The result is npub_argmax_rows over the concatenated vocabulary. */
int npub_argmax_keys(const void* x, int64_t ldx, int rows, int cols, int32_t index_offset, uint64_t* keys,
                     void* stream);
int npub_select_keys(const uint64_t* keys, int ranks, int rows, int32_t* ids, void* stream);

/* -------------------------------------------------------- attention ----
 * Causal prefill attention, llama_layer.py:114-137, legalize.py:117-127 for
 * every sequence b and head h: S = Q K^T * scale + mask; P = softmax(S); O = P V.
 * q, k, v: fp16 rows of `batch` sequences of `tokens` rows each (sequence b at
 * rows [b*tokens, (b+1)*tokens)), row strides ldq/ldk/ldv; head h reads
 * columns [h*head_dim, (h+1)*head_dim) of q and kv head h / (heads/kv_heads)
 * of k and v (grouped-query heads).  out fp16 [batch*tokens, heads*head_dim] (ldo).
 * head_dim % 16 == 0, head_dim <= 256; batch*heads <= 65535.  head_dim 128 runs a
 * fused flash-attention kernel and needs no scratch; other sizes materialise
 * S/P: npub_attention_workspace() bytes, 256-byte aligned. */
int npub_attention_prefill(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                           void* out, int64_t ldo, int batch, int tokens, int heads, int kv_heads, int head_dim,
                           float scale, int causal, void* workspace, size_t workspace_bytes, void* stream);
size_t npub_attention_workspace(int batch, int tokens, int heads, int head_dim);

/* Decode attention over a KV cache (one new query token per sequence):
 *   out[b, h, :] = softmax(q[b,h,:] . K[b, kvh, :len[b], :]^T * scale) V[b, kvh, :len[b], :]
 * q fp16 [batch, heads*head_dim] (ldq); caches fp16 [batch, kv_heads, cap, head_dim]
 * (contiguous per head); lens int32 [batch] (NULL = all `ctx_len`).
 * head_dim == 128.  Flash-decoding split over the context; scratch:
 * npub_attention_decode_workspace(). */
int npub_attention_decode(const void* q, int64_t ldq, const void* k_cache, const void* v_cache, int64_t cap,
                          const int32_t* lens, int ctx_len, void* out, int64_t ldo, int batch, int heads,
                          int kv_heads, int head_dim, float scale, void* workspace, size_t workspace_bytes,
                          void* stream);
size_t npub_attention_decode_workspace(int batch, int heads, int ctx_len, int head_dim);

/* Append one token's K and V rows per sequence to the caches at position
 * pos[b] (or pos0 when pos is NULL): cache[b, h, pos, :] = src[b, h*hd : (h+1)*hd]. */
int npub_kv_append(const void* k_new, int64_t ldk, const void* v_new, int64_t ldv, void* k_cache, void* v_cache,
                   int64_t cap, const int32_t* pos, int pos0, int batch, int kv_heads, int head_dim, void* stream);

/* Decode-step RoPE fused with the KV-cache append (the rope_Q / rope_Kt macros,
 * llama_layer.py:96-112, plus the cache write of a decode step, which the
 * reference does not have).  qkv [tokens, ldx] fp16 holds q heads, then k
 * heads, then v heads (head_dim columns each); q and k are rotated in place
 * with the positions[t] of each row (the same arithmetic as npub_rope), and
 * the rotated k and the v heads are written to k_cache / v_cache
 * [tokens, kv_heads, cap, head_dim] at slot positions[t].  lens (may be NULL)
 * receives positions[t] + 1.  head_dim % 16 == 0, <= 512; 16-byte aligned. */
int npub_rope_kv_append(void* qkv, int64_t ldx, int tokens, int q_heads, int kv_heads, int head_dim,
                        const int32_t* positions, float theta, void* k_cache, void* v_cache, int64_t cap,
                        int32_t* lens, void* stream);

/* Prompt counterpart of npub_rope_kv_append (prefill; the reference rotates
 * q and k with the same macros, llama_layer.py:96-112, and keeps no cache).
 * qkv holds tokens = batch * tokens_per_seq rows, row r belonging to sequence
 * r / tokens_per_seq; q and k are rotated in place with positions[r], and the
 * rotated k and the v heads are written to k_cache / v_cache
 * [batch, kv_heads, cap, head_dim] at slot positions[r].  A row whose
 * position lies outside [0, cap) is rotated but not stored.  One kernel in
 * place of npub_rope and two strided cache copies. */
int npub_rope_kv_store(void* qkv, int64_t ldx, int tokens, int tokens_per_seq, int q_heads, int kv_heads,
                       int head_dim, const int32_t* positions, float theta, void* k_cache, void* v_cache, int64_t cap,
                       void* stream);

/* RoPE with a frequency table instead of theta (the Llama-3.2 layer of
 * d_compiler/npu_compiler/model.py:20-21: base 500000 with the frequency
 * scaling of legalize.py:50-64, rope_tables(..., llama3_scaling=True) at
 * legalize.py:67-76).  inv_freq: device fp32 [head_dim/2], frequency i of every
 * head; angle = p * inv_freq[i].  Otherwise as npub_rope, npub_rope_kv_append
 * and npub_rope_kv_store. */
int npub_rope_freqs(void* x, int64_t ldx, int tokens, int heads, int head_dim, const int32_t* positions, int pos0,
                    const float* inv_freq, void* stream);
int npub_rope_kv_append_freqs(void* qkv, int64_t ldx, int tokens, int q_heads, int kv_heads, int head_dim,
                              const int32_t* positions, const float* inv_freq, void* k_cache, void* v_cache,
                              int64_t cap, int32_t* lens, void* stream);
int npub_rope_kv_store_freqs(void* qkv, int64_t ldx, int tokens, int tokens_per_seq, int q_heads, int kv_heads,
                             int head_dim, const int32_t* positions, const float* inv_freq, void* k_cache,
                             void* v_cache, int64_t cap, void* stream);
/* The table itself, on the host (out: float [head_dim/2]): theta^(-2i/head_dim),
 * scaled as legalize.py:50-64 (_llama3_scale_freqs: factor, low, high,
 * old_ctx = 32, 1, 4, 8192 there) when factor > 0; factor <= 0 gives the
 * unscaled table.  Computed in double precision, rounded to float. */
int npub_rope_llama3_freqs(float* out, int head_dim, double theta, double factor, double low, double high,
                           double old_ctx);

/* ------------------------------------------------- NPU ISA semantics ----
 * One compute instruction of the NPU over PE buffers (_poc/mysim.cpp:114-141):
 * `word` is the 32-bit instruction (opcodes 0x01-0x13 vector, 0x40-0x43
 * matrix elementwise; 0x42 with mode 2 is the matrix multiply and is not
 * taken here).  in1/in2/prev_out/out are fp32 device arrays of n elements
 * (in2 read only in vector mode; prev_out is the previous PE output, read by
 * mul-add 0x0C).  Float32 arithmetic as the cmodel does it; logical, shift,
 * compare and convert results are bit-exact with the cmodel on x86-64. */
int npub_isa_vector(uint32_t word, const float* in1, const float* in2, const float* prev_out, float* out, int64_t n,
                    void* stream);
/* The cmodel's store rounding (mysim.cpp:19-38, applied by save 0x98):
 * fp32 -> fp16 round-to-nearest-even, NaN -> sign|0x7C00|0x200. */
int npub_f32_to_f16(const float* x, uint16_t* y, int64_t n, void* stream);
/* fp16 -> fp32 (the cmodel's load of the G-buffer). */
int npub_f16_to_f32(const uint16_t* x, float* y, int64_t n, void* stream);

/* ------------------------------------------------------------ programs --
 * Whole NPU programs on the GPU: the drop-in for run(asm, gbuf, gn, rundir,
 * maxrun) of b_program_examples/npu.py:62-71 and run(program, gbuf, gn,
 * maxrun) of d_compiler/npu_compiler/runtime.py:46-77, which write
 * program_memory.bin and G_buffer_data.bin and run the cmodel
 * (_poc/mysim.cpp:42-157) on them.
 *
 * npub_program_create decodes words[0 .. nwords) on the host -- at most
 * maxrun program-counter steps, HALT (0xFF) ends the program, words past the
 * end are NOPs, g_in is the number of G-buffer words the caller will pass --
 * into tasks in dependency order.  It returns NPUB_ERR_INVALID_ARG when an
 * instruction would read past a PE input buffer (undefined behaviour in the
 * cmodel); npub_program_error_pc() then gives its program counter (this
 * thread's last failed create).  npub_program_load copies the task tables
 * into a caller workspace of npub_program_workspace() bytes (256-byte
 * aligned; synchronises the stream).  npub_program_run executes the program
 * on the G-buffer g_in [n_in] (fp16, device; n_in <= the g_in given to
 * create) and writes the first gn words of the final G-buffer to g_out (fp16,
 * device; words the machine never held read +0), which is the cmodel's
 * --gout write-back.  A run may follow a load any number of times.
 * Results are the cmodel's bits (float32 arithmetic without contraction,
 * the matmul's ascending-k accumulation, x86-64 integer conversions, fp16
 * store rounding), except exp (0x0F) and the matrix activation x^2 sigmoid(x)
 * (CUDA's expf: a few float32 ulps from the host libm before the fp16 store).
 * npub_program_info fills up to 7 counts: steps executed, tasks, levels,
 * G-buffer words, temporary words, work chunks, CTAs of the run. */
int npub_program_create(const uint32_t* words, int64_t nwords, int64_t maxrun, int64_t g_in, void** program);
int npub_program_error_pc(void);
int npub_program_info(const void* program, int64_t* info, int n);
size_t npub_program_workspace(const void* program);
int npub_program_load(const void* program, void* workspace, size_t workspace_bytes, void* stream);
int npub_program_run(const void* program, const uint16_t* g_in, int64_t n_in, uint16_t* g_out, int64_t gn,
                     void* workspace, size_t workspace_bytes, void* stream);
int npub_program_destroy(void* program);

/* ---------------------------------------------- tensor-parallel all-reduce --
 * One-shot fp16 all-reduce over NVLink peer memory for the decode-sized
 * reductions after the row-parallel O and down projections (the TP sharding
 * of the layer; the single-NPU reference has no counterpart).  Set-up: every
 * rank calls npub_comm_create (allocates 2 x max_bytes of IPC-shareable
 * staging plus flags; writes npub_comm_handle_bytes() bytes of handle), the
 * handles are all-gathered in rank order by the caller (e.g. torch.distributed),
 * then npub_comm_open maps the peers.  npub_allreduce_f16 sums n fp16 elements
 * (n % 8 == 0, n * 2 <= max_bytes, 16-byte aligned; in may equal out) over
 * the ranks in rank order with fp32 accumulation: every rank gets the same
 * bits.  All ranks must make the same sequence of calls; waits on peers are
 * bounded (2 s) and report NPUB_ERR_DEVICE_TIMEOUT through npub_device_error. */
size_t npub_comm_handle_bytes(void);
int npub_comm_create(int world, int rank, size_t max_bytes, void** comm, void* handle_out);
int npub_comm_open(void* comm, const void* all_handles);
int npub_allreduce_f16(void* comm, const void* in, void* out, int64_t n, void* stream);
/* The same sum of a [rows, d] message (d % 32 == 0) with the residual add and
 * the next RMSNorm's inputs folded in (llama_layer.py:139-141 after the TP
 * reduction): out = fp16(fp16(sum) + residual), G = fp16(out * gamma) and
 * ss[(c/32)*ss_ld + r] = sum over the 32 columns c.. of out[r, c]^2 -- the
 * rs_part of npub_w8a16_gemm_rms. */
int npub_allreduce_f16_rms(void* comm, const void* in, void* out, int rows, int d, const void* residual,
                           const void* gamma, void* G, float* ss, int64_t ss_ld, void* stream);
int npub_comm_destroy(void* comm);
#ifdef __cplusplus
}
#endif
#endif /* NPUB_H */

/*
 * isa_oracle.c -- CPU restatement of the NPU cmodel's instruction semantics.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA path: only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.
 * Nothing in npu_comp_b200/ links or calls it.
 *
 * It restates, in fresh code, the behaviour of the reference simulator
 * `_poc/mysim.cpp` (KwanyoungCho/NPU_COMP):
 *   - fp16 <-> fp32 conversion (mysim.cpp:19-38): round-to-nearest-even,
 *     subnormals kept, overflow to inf, NaN stored as sign|0x7C00|0x200;
 *   - the fetch/decode/execute loop (mysim.cpp:83-145) over a flat fp16
 *     G-buffer that grows on demand (mysim.cpp:58), float32 compute with an
 *     fp16 round only on `save` (mysim.cpp:102-104);
 *   - the stdout trace format (mysim.cpp:69-75, 87-88, 100-104, 142-144), so
 *     that the golden traces under `_poc/goldens/` pin this restatement byte
 *     for byte;
 *   - the G-buffer write-back of `--gout` (mysim.cpp:147-155).
 * Integer-valued operations (logical 0x08, shift 0x09, compare 0x11,
 * convert 0x13) follow x86-64 conversion behaviour for out-of-range values,
 * which is what the reference binary does on its host.
 *
 * Build: gcc -O2 -ffp-contract=off -fPIC -shared isa_oracle.c -o libisa_oracle.so -lm
 * (oracle/Makefile).  -ffp-contract=off keeps a*b+c as two roundings, like
 * the reference build on x86-64 without FMA.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ fp16 */

uint16_t ora_f32_to_f16(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    uint32_t e = (u >> 23) & 0xFFu, m = u & 0x7FFFFFu;
    if (e == 0xFFu) return (uint16_t)(sign | 0x7C00u | (m ? 0x200u : 0u));
    int he = (int)e - 112; /* exponent rebased from bias 127 to bias 15 */
    if (he >= 31) return (uint16_t)(sign | 0x7C00u);
    if (he <= 0) {
        if (he < -10) return sign; /* below half the smallest subnormal */
        m |= 0x800000u;
        int shift = 14 - he;
        uint32_t q = m >> shift, r = m & ((1u << shift) - 1u), halfway = 1u << (shift - 1);
        if (r > halfway || (r == halfway && (q & 1u))) q++;
        return (uint16_t)(sign | q); /* q == 0x400 encodes the smallest normal */
    }
    uint32_t out = ((uint32_t)he << 10) + (m >> 13), r = m & 0x1FFFu;
    if (r > 0x1000u || (r == 0x1000u && (out & 1u))) out++; /* carry may reach inf */
    return (uint16_t)(sign | out);
}

float ora_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            int sh = 0;
            while (!(m & 0x400u)) { m <<= 1; sh++; }
            bits = sign | ((uint32_t)(113 - sh) << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static inline float round_f16(float x) { return ora_f16_to_f32(ora_f32_to_f16(x)); }

/* x86-64 cvttss2si semantics: truncate, out-of-range and NaN give INT64_MIN. */
static inline int64_t to_i64(float a) {
    if (!(fabsf(a) < 9.2233720368547758e18f)) return INT64_MIN;
    return (int64_t)a;
}
static inline int32_t to_i32(float a) {
    if (!(fabsf(a) < 2147483648.0f)) return INT32_MIN;
    return (int32_t)a;
}

/* SSE NaN results, whatever operand order this compiler picks for a
 * commutative operation: a NaN operand comes back made quiet; an invalid
 * operation on non-NaN operands gives the indefinite NaN 0xFFC00000.  When
 * both operands are NaN, the one the reference simulator's compiled code
 * keeps in the destination register wins (measured against it): the left
 * operand of a op b, the product in mul-add, the running sum in the matmul,
 * and in the activation the sigmoid after a matmul, x * x after an
 * elementwise matrix op. */
static inline float quietf(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    u |= 0x00400000u;
    memcpy(&x, &u, 4);
    return x;
}
static inline float sse2(float r, float x, float y) {
    if (r == r) return r;
    if (x != x) return quietf(x);
    if (y != y) return quietf(y);
    uint32_t u = 0xFFC00000u;
    memcpy(&r, &u, 4);
    return r;
}
static inline float f_add(float x, float y) { return sse2(x + y, x, y); }
static inline float f_sub(float x, float y) { return sse2(x - y, x, y); }
static inline float f_mul(float x, float y) { return sse2(x * y, x, y); }
static inline float f_div(float x, float y) { return sse2(x / y, x, y); }

static inline float hw_act(float x, int sigmoid_first) { /* x^2 * sigmoid(x) (mysim.cpp:39-40) */
    float e = expf(-x);
    float s = f_div(1.0f, f_add(1.0f, e));
    float xx = f_mul(x, x);
    return sigmoid_first ? f_mul(s, xx) : f_mul(xx, s);
}

/* --------------------------------------------------------------- buffers */

typedef struct {
    float* v;
    long n, cap;
} fvec;

static int fvec_resize(fvec* a, long n) {
    if (n > a->cap) {
        long c = n < 16 ? 16 : n;
        float* p = (float*)realloc(a->v, (size_t)c * sizeof(float));
        if (!p) return -1;
        a->v = p;
        a->cap = c;
    }
    a->n = n;
    return 0;
}

typedef struct {
    char* s;
    long n, cap;
    int on;
} tbuf;

static void tput(tbuf* t, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
#include <stdarg.h>
static void tput(tbuf* t, const char* fmt, ...) {
    if (!t->on) return;
    for (;;) {
        va_list ap;
        va_start(ap, fmt);
        long room = t->cap - t->n;
        int k = vsnprintf(t->s + t->n, (size_t)(room > 0 ? room : 0), fmt, ap);
        va_end(ap);
        if (k < 0) return;
        if (k < room) { t->n += k; return; }
        long c = t->cap * 2 + k + 4096;
        char* p = (char*)realloc(t->s, (size_t)c);
        if (!p) { t->on = 0; return; }
        t->s = p;
        t->cap = c;
    }
}

typedef struct {
    float* g; /* G-buffer values, always fp16-representable */
    long gsize;
    long gin_n;
    fvec in1, in2, out;
    uint32_t blo[3], bhi[3];
    long vlen, tA[2], tB[2];
    tbuf tr;
    long executed;
    int error; /* 1: operand read past a PE buffer, 2: allocation failure */
} ora_state;

static int ensure_g(ora_state* st, long idx) {
    if (idx < st->gsize) return 0;
    long ns = idx + 1024;
    float* p = (float*)realloc(st->g, (size_t)ns * sizeof(float));
    if (!p) return -1;
    memset(p + st->gsize, 0, (size_t)(ns - st->gsize) * sizeof(float));
    st->g = p;
    st->gsize = ns;
    return 0;
}

/* Create a machine whose G-buffer holds `gin_n` fp16 words (capacity at least gcap). */
void* ora_create(const uint16_t* gin, long gin_n, long gcap) {
    ora_state* st = (ora_state*)calloc(1, sizeof(ora_state));
    if (!st) return NULL;
    long n = gcap > gin_n ? gcap : gin_n;
    if (n < 1) n = 1;
    st->g = (float*)calloc((size_t)n, sizeof(float));
    if (!st->g) { free(st); return NULL; }
    st->gsize = n;
    st->gin_n = gin_n;
    for (long i = 0; i < gin_n; i++) st->g[i] = ora_f16_to_f32(gin[i]);
    return st;
}

void ora_destroy(void* h) {
    ora_state* st = (ora_state*)h;
    if (!st) return;
    free(st->g); free(st->in1.v); free(st->in2.v); free(st->out.v); free(st->tr.s);
    free(st);
}

static float operand_b(ora_state* st, int mode, int cst, long i) {
    if (mode == 2) {
        if (i >= st->in2.n) { st->error = 1; return 0.0f; }
        return st->in2.v[i];
    }
    return (float)cst;
}

/* Whether an opcode reads its second operand (sqrt, exp and convert do not). */
static int reads_b(uint32_t op) { return !(op == 0x0Eu || op == 0x0Fu || op == 0x13u); }

/* One element of a compute instruction (mysim.cpp:117-140): a from PE input
 * 1, b the second operand (PE input 2 in vector mode, else the immediate),
 * prev the previous PE output (read by mul-add). */
static float elem_op(uint32_t w, float a, float b, float prev) {
    uint32_t op = w & 0xFFu;
    int mode = (int)((w >> 30) & 3u), actf = (int)((w >> 29) & 1u);
    int matrix = op >= 0x40u && op <= 0x43u;
    int cst = (int)((w >> 8) & 0xFFFFu);
    float r = a;
    switch (op) {
        case 0x01: case 0x40: r = f_add(a, b); break;
        case 0x02: case 0x41: r = f_sub(a, b); break;
        case 0x0A: case 0x42: r = f_mul(a, b); break;
        case 0x0B: r = f_div(a, b); break;
        case 0x0C: r = f_add(f_mul(a, b), prev); break;
        case 0x0D: case 0x43: r = b; break;
        case 0x0E: r = sqrtf(a); break;
        case 0x0F: r = expf(a); break;
        case 0x11: r = (a == b) ? 1.0f : 0.0f; break;
        case 0x12: r = ((w >> 28) & 1u) ? (a > b ? a : b) : (a < b ? a : b); break;
        case 0x13: r = (float)to_i64(a); break;
        case 0x09: {
            int16_t s = (int16_t)cst;
            if (mode == 2) s = (int16_t)to_i32(b);
            r = f_mul(a, ldexpf(1.0f, (int)s));
        } break;
        case 0x08: {
            int64_t ia = to_i64(a), ib = to_i64(b);
            switch ((w >> 27) & 7u) {
                case 0: r = (float)(ia & ib); break;
                case 1: r = (float)(ia | ib); break;
                case 2: r = (float)(~ia); break;
                case 3: r = (float)(ia ^ ib); break;
                case 4: r = (float)(~(ia & ib)); break;
                case 5: r = (float)(~(ia | ib)); break;
                default: break;
            }
        } break;
        default: break;
    }
    if (actf && matrix) r = hw_act(r, 0);
    return r;
}

/* Elementwise semantics of one compute instruction over fp32 PE buffers
 * (in2 is read in vector mode only, prev by mul-add); the checker for the
 * GPU's npub_isa_vector. */
void ora_vector(uint32_t w, const float* in1, const float* in2, const float* prev, float* out, long n) {
    int mode = (int)((w >> 30) & 3u);
    int cst = (int)((w >> 8) & 0xFFFFu);
    for (long i = 0; i < n; i++) {
        float b = mode == 2 ? in2[i] : (float)cst;
        out[i] = elem_op(w, in1[i], b, prev ? prev[i] : 0.0f);
    }
}

/*
 * Execute up to `maxrun` instructions of `prog` (nprog words).  When `trace`
 * is non-zero the reference's stdout trace is reproduced; `gbytes`/`pbytes`
 * are the byte sizes of the two input files (with their trailing newline),
 * which only appear in the trace header.  Returns the number of program
 * counter steps taken, or -1 on a machine error (see ora_error).
 */
long ora_exec(void* h, const uint32_t* prog, long nprog, long maxrun, int trace, long gbytes, long pbytes) {
    ora_state* st = (ora_state*)h;
    st->tr.on = trace;
    st->tr.n = 0;
    tput(&st->tr, "G_buffer size :  %ld\n\n\n\n", gbytes);
    tput(&st->tr, "0\n");
    tput(&st->tr, "Program memory size :  %lx\n\n\n\n", pbytes);
    tput(&st->tr, "0\n");
    for (int k = 0; k < 20; k++) tput(&st->tr, "%x\n", k < nprog ? prog[k] : 0u);
    tput(&st->tr, "\n\n\n");

    long pc;
    for (pc = 0; pc < maxrun; pc++) {
        uint32_t w = pc < nprog ? prog[pc] : 0u;
        uint32_t op = w & 0xFFu;
        int mode = (int)((w >> 30) & 3u);
        int actf = (int)((w >> 29) & 1u);
        tput(&st->tr, "p_counter :  %ld\n", pc);
        tput(&st->tr, "instruction :  %x\n", w);
        if (op == 0xFFu) { tput(&st->tr, "HALT --- \n\n\n\n"); pc++; break; }
        if (w == 0) {
            tput(&st->tr, "NOP --- \n");
        } else if (op == 0x80u) { /* set address: operand select, hi/lo half */
            int o = (int)((w >> 30) & 3u);
            uint32_t v = (w >> 8) & 0xFFFFu;
            if (o < 3) { if ((w >> 29) & 1u) st->bhi[o] = v; else st->blo[o] = v; }
        } else if (op == 0x82u) {
            st->vlen = (long)((w >> 8) & 0xFFFFu);
        } else if (op == 0x88u) {
            int sel = (int)((w >> 31) & 1u);
            st->tA[sel] = (long)((w >> 8) & 0xFFu);
            st->tB[sel] = (long)((w >> 16) & 0xFFu);
        } else if (op == 0x90u) { /* load G -> PE input buffer */
            int matrix = (int)((w >> 31) & 1u), sel = (int)((w >> 30) & 1u);
            long base = (long)(st->blo[sel] | (st->bhi[sel] << 16));
            long n = matrix ? st->tA[sel] * st->tB[sel] : st->vlen;
            fvec* d = sel == 0 ? &st->in1 : &st->in2;
            if (fvec_resize(d, n) || ensure_g(st, base + n)) { st->error = 2; return -1; }
            for (long i = 0; i < n; i++) d->v[i] = st->g[base + i];
            const char* lbl = sel == 0 ? "PE_in_data_1_array :  " : "PE_in_data_2_array :  ";
            for (long i = 0; i < n; i++) tput(&st->tr, "%s%g\n", lbl, (double)d->v[i]);
        } else if (op == 0x98u) { /* save PE output -> G, fp16 round */
            long base = (long)(st->blo[2] | (st->bhi[2] << 16));
            long n = st->out.n;
            if (ensure_g(st, base + n)) { st->error = 2; return -1; }
            for (long i = 0; i < n; i++) st->g[base + i] = round_f16(st->out.v[i]);
            for (long i = 0; i < n; i++) tput(&st->tr, "PE_out_array :  %g\n", (double)st->out.v[i]);
        } else { /* compute, float32 */
            int matrix = op >= 0x40u && op <= 0x43u;
            int cst = (int)((w >> 8) & 0xFFFFu);
            if (matrix && op == 0x42u && mode == 2) {
                long rA = st->tA[0], cA = st->tB[0], cB = st->tB[1];
                if (st->in1.n < rA * cA || st->in2.n < cA * cB) { st->error = 1; return -1; }
                if (fvec_resize(&st->out, rA * cB)) { st->error = 2; return -1; }
                for (long i = 0; i < rA; i++)
                    for (long j = 0; j < cB; j++) {
                        float acc = 0.0f;
                        for (long k = 0; k < cA; k++) acc = f_add(acc, f_mul(st->in1.v[i * cA + k], st->in2.v[k * cB + j]));
                        st->out.v[i * cB + j] = actf ? hw_act(acc, 1) : acc;
                    }
            } else {
                long n = matrix ? st->tA[0] * st->tB[0] : st->vlen;
                if (st->out.n != n) {
                    if (fvec_resize(&st->out, n)) { st->error = 2; return -1; }
                    memset(st->out.v, 0, (size_t)n * sizeof(float));
                }
                if (st->in1.n < n) { st->error = 1; return -1; }
                const int rb = reads_b(op);
                for (long i = 0; i < n; i++) {
                    float b = rb ? operand_b(st, mode, cst, i) : 0.0f;
                    st->out.v[i] = elem_op(w, st->in1.v[i], b, st->out.v[i]);
                }
                if (st->error) return -1;
            }
            for (long i = 0; i < st->out.n; i++) tput(&st->tr, "%g\n", (double)st->out.v[i]);
        }
        tput(&st->tr, "\n\n\n");
    }
    st->executed = pc;
    return pc;
}

int ora_error(void* h) { return ((ora_state*)h)->error; }
long ora_trace_len(void* h) { return ((ora_state*)h)->tr.n; }
const char* ora_trace(void* h) { return ((ora_state*)h)->tr.s; }
long ora_gsize(void* h) { return ((ora_state*)h)->gsize; }

/* fp16 image of G[0..n): entries past the buffer read as +0 (mysim.cpp:151). */
void ora_gread(void* h, uint16_t* out, long n) {
    ora_state* st = (ora_state*)h;
    for (long i = 0; i < n; i++) out[i] = ora_f32_to_f16(i < st->gsize ? st->g[i] : 0.0f);
}

/* Bulk fp32 -> fp16 conversion with the cmodel's rounding (for numpy-side checks). */
void ora_f32_to_f16_array(const float* x, uint16_t* y, long n) {
    for (long i = 0; i < n; i++) y[i] = ora_f32_to_f16(x[i]);
}

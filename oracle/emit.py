"""NPU program emitter -- TEST INFRASTRUCTURE ONLY (the checker).

numpy-only restatement of the reference's instruction encoder
(b_program_examples/npu.py:10-38; the same words as
d_compiler/npu_compiler/isa.py) and of the program shapes the reference
emits, so that oracle programs can be built without TVM:
  * one-shot matmul macro            b_program_examples/npu.py:41-47
  * 64-tiled matmul (fp16 K-partial
    accumulation, gather/scatter)    d_compiler/npu_compiler/codegen.py:59-108
  * chunked elementwise (<= 8192)    d_compiler/npu_compiler/codegen.py:160-177
  * vec/unary macros and the RMSNorm,
    SiLU/SwiGLU, softmax and RoPE
    recipes                          b_program_examples/llama_layer.py:71-112,
                                     test_rmsnorm.py:33-43, test_swiglu.py:28-40,
                                     test_attention.py:42-55
The instruction word format (field positions) is fixed by the NPU ISA
(_poc/README.md:69-114), so it is necessarily the same as the reference's.
"""
from __future__ import annotations

from typing import List

import numpy as np

# opcodes (_poc/README.md:84-114, mysim.cpp:89-141)
OP = {
    "add": 0x01, "sub": 0x02, "logic": 0x08, "shift": 0x09, "mul": 0x0A, "div": 0x0B, "muladd": 0x0C,
    "move": 0x0D, "sqrt": 0x0E, "exp": 0x0F, "cmp": 0x11, "minmax": 0x12, "cvt": 0x13,
    "m_add": 0x40, "m_sub": 0x41, "m_mul": 0x42, "m_move": 0x43,
    "addr": 0x80, "vlen": 0x82, "tile": 0x88, "load": 0x90, "save": 0x98, "halt": 0xFF,
}
SRC1, SRC2, DST = 0, 1, 2
IMM, SCALAR, VECTOR = 0, 1, 2


class Asm:
    """Collects 32-bit NPU instruction words."""

    def __init__(self):
        self.words: List[int] = []

    def emit(self, w: int) -> None:
        self.words.append(int(w) & 0xFFFFFFFF)

    # control / data movement
    def halt(self):
        self.emit(OP["halt"])

    def nop(self):
        self.emit(0)

    def addr(self, operand: int, a: int):
        for half, v in ((0, a & 0xFFFF), (1, (a >> 16) & 0xFFFF)):
            self.emit((operand << 30) | (half << 29) | (v << 8) | OP["addr"])

    def vlen(self, n: int):
        self.emit(((n & 0xFFFF) << 8) | OP["vlen"])

    def tile(self, matrix: int, rows: int, cols: int):
        self.emit((matrix << 31) | ((cols & 0xFF) << 16) | ((rows & 0xFF) << 8) | OP["tile"])

    def load(self, matrix: int, operand: int):
        self.emit((matrix << 31) | (operand << 30) | OP["load"])

    def save(self, matrix: int):
        self.emit((matrix << 31) | OP["save"])

    # compute
    def compute(self, name: str, mode: int = VECTOR, imm: int = 0, act: bool = False, bit28: int = 0, sub: int = 0):
        self.emit((mode << 30) | ((1 if act else 0) << 29) | (bit28 << 28) | (sub << 27) | ((imm & 0xFFFF) << 8)
                  | OP[name])

    def v_add(self, mode=VECTOR, imm=0): self.compute("add", mode, imm)
    def v_sub(self, mode=VECTOR, imm=0): self.compute("sub", mode, imm)
    def v_mul(self, mode=VECTOR, imm=0): self.compute("mul", mode, imm)
    def v_div(self, mode=VECTOR, imm=0): self.compute("div", mode, imm)
    def v_muladd(self, mode=VECTOR, imm=0): self.compute("muladd", mode, imm)
    def v_move(self, mode=VECTOR, imm=0): self.compute("move", mode, imm)
    def v_sqrt(self): self.compute("sqrt", IMM)
    def v_exp(self): self.compute("exp", IMM)
    def v_max(self, mode=VECTOR, imm=0): self.compute("minmax", mode, imm, bit28=1)
    def v_min(self, mode=VECTOR, imm=0): self.compute("minmax", mode, imm, bit28=0)
    def m_add(self, mode=VECTOR, imm=0, act=False): self.compute("m_add", mode, imm, act)
    def m_mul(self, mode=VECTOR, imm=0, act=False): self.compute("m_mul", mode, imm, act)

    def bytes(self) -> bytes:
        return np.asarray(self.words, dtype="<u4").tobytes() + b"\n"


class GBuf:
    """Bump allocator over an fp16 G-buffer image (b_program_examples/npu.py:49-60)."""

    def __init__(self, size: int = 1 << 16):
        self.mem = np.zeros(size, dtype=np.float16)
        self.top = 0

    def alloc(self, n: int) -> int:
        a = self.top
        self.top += int(n)
        if self.top > self.mem.size:
            grown = np.zeros(max(self.top, 2 * self.mem.size), dtype=np.float16)
            grown[: self.mem.size] = self.mem
            self.mem = grown
        return a

    def put(self, addr: int, values) -> None:
        v = np.asarray(values, dtype=np.float32).reshape(-1).astype(np.float16)
        self.mem[addr: addr + v.size] = v

    def image(self, count: int) -> np.ndarray:
        return self.mem[:count].copy()


# ------------------------------------------------------------------ macros

def matmul(a: Asm, A: int, B: int, C: int, M: int, K: int, N: int, act: bool = False) -> None:
    """One-shot C[M,N] = A[M,K] @ B[K,N] (npu.py:41-47); dims <= 255."""
    a.tile(0, M, K)
    a.tile(1, K, N)
    a.addr(SRC1, A)
    a.addr(SRC2, B)
    a.load(1, 0)
    a.load(1, 1)
    a.m_mul(mode=VECTOR, act=act)
    a.addr(DST, C)
    a.save(1)


def copy2d(a: Asm, dst: int, dst_stride: int, src: int, src_stride: int, rows: int, cols: int) -> None:
    for r in range(rows):
        a.vlen(cols)
        a.addr(SRC1, src + r * src_stride)
        a.load(0, 0)
        a.v_add(mode=IMM, imm=0)
        a.addr(DST, dst + r * dst_stride)
        a.save(0)


def matmul_tiled(a: Asm, A: int, B: int, C: int, M: int, K: int, N: int, scratch: int, T: int = 64) -> None:
    """64-tiled matmul as codegen.py:59-108 emits it.  scratch holds 4*T*T words
    (gathered A tile, gathered B tile, partial product, output accumulator).
    Numerically C = fp16(C + fp16(A_k @ B_k)) per K tile (test_tiling.py:37-47)."""
    sA, sB, sP, sC = scratch, scratch + T * T, scratch + 2 * T * T, scratch + 3 * T * T
    for mi in range(0, M, T):
        mt = min(T, M - mi)
        for nj in range(0, N, T):
            nt = min(T, N - nj)
            cdst = (C + mi * N) if nt == N else sC
            for ti, kk in enumerate(range(0, K, T)):
                kt = min(T, K - kk)
                if kt == K:
                    a_src = A + mi * K
                else:
                    copy2d(a, sA, kt, A + mi * K + kk, K, mt, kt)
                    a_src = sA
                if nt == N:
                    b_src = B + kk * N
                else:
                    copy2d(a, sB, nt, B + kk * N + nj, N, kt, nt)
                    b_src = sB
                a.tile(0, mt, kt)
                a.tile(1, kt, nt)
                a.addr(SRC1, a_src)
                a.load(1, 0)
                a.addr(SRC2, b_src)
                a.load(1, 1)
                a.m_mul(mode=VECTOR)
                if ti == 0:
                    a.addr(DST, cdst)
                    a.save(1)
                else:
                    a.addr(DST, sP)
                    a.save(1)
                    a.vlen(mt * nt)
                    a.addr(SRC1, cdst)
                    a.load(0, 0)
                    a.addr(SRC2, sP)
                    a.load(0, 1)
                    a.v_add(mode=VECTOR)
                    a.addr(DST, cdst)
                    a.save(0)
            if nt != N:
                copy2d(a, C + mi * N + nj, N, sC, nt, mt, nt)


def ew(a: Asm, name: str, dst: int, src1: int, src2=None, n: int = 0, chunk: int = 8192, mode: int = VECTOR,
       imm: int = 0) -> None:
    """Elementwise op over n contiguous words, chunked (codegen.py:160-177)."""
    for base in range(0, n, chunk):
        m = min(chunk, n - base)
        a.vlen(m)
        a.addr(SRC1, src1 + base)
        a.load(0, 0)
        if src2 is not None and mode == VECTOR:
            a.addr(SRC2, src2 + base)
            a.load(0, 1)
        if name in ("sqrt", "exp"):
            a.compute(name, IMM)
        else:
            a.compute(name, mode, imm)
        a.addr(DST, dst + base)
        a.save(0)


# ------------------------------------------------------- program builders

def w8a16_program(A: np.ndarray, Wd: np.ndarray, T: int = 64):
    """G-buffer image + tiled program for C = A @ Wd, where Wd [K, N] holds the
    dequantised weights fp16(q * s) (the W8A16 matmul run on the NPU's fp16
    datapath).  Returns (words, gbuf_image, c_addr, gn)."""
    M, K = A.shape
    K2, N = Wd.shape
    assert K == K2
    g = GBuf(M * K + K * N + M * N + 4 * T * T)
    aA = g.alloc(M * K)
    g.put(aA, A)
    aB = g.alloc(K * N)
    g.put(aB, Wd)
    aC = g.alloc(M * N)
    scr = g.alloc(4 * T * T)
    a = Asm()
    if max(M, K, N) <= 255 and T is None:
        matmul(a, aA, aB, aC, M, K, N)
    else:
        matmul_tiled(a, aA, aB, aC, M, K, N, scr, T)
    a.halt()
    return a.words, g.image(g.top), aC, g.top


def rmsnorm_program(X: np.ndarray, w: np.ndarray):
    """Per-token RMSNorm recipe of test_rmsnorm.py:33-43 / llama_layer.py:79-89
    (eps = 0: the integer immediate cannot encode it).  Rows of <= 255 words."""
    S, D = X.shape
    g = GBuf()
    aX = g.alloc(S * D); g.put(aX, X)
    aW = g.alloc(D); g.put(aW, w)
    aOne = g.alloc(D); g.put(aOne, np.ones(D))
    aOut = g.alloc(S * D)
    aSq = g.alloc(D); aSS = g.alloc(1); aMean = g.alloc(1); aRms = g.alloc(1); aInv = g.alloc(1)
    aScale = g.alloc(D); aTmp = g.alloc(S * D)
    a = Asm()

    def vec(name, s1, s2, dst, n, mode=VECTOR, imm=0):
        a.vlen(n); a.addr(SRC1, s1); a.load(0, 0)
        if mode == VECTOR:
            a.addr(SRC2, s2); a.load(0, 1)
        a.compute(name, mode, imm); a.addr(DST, dst); a.save(0)

    for t in range(S):
        xt = aX + t * D
        vec("mul", xt, xt, aSq, D)
        matmul(a, aSq, aOne, aSS, 1, D, 1)
        vec("div", aSS, 0, aMean, 1, mode=IMM, imm=D)
        a.vlen(1); a.addr(SRC1, aMean); a.load(0, 0); a.v_sqrt(); a.addr(DST, aRms); a.save(0)
        vec("div", aOne, aRms, aInv, 1)
        matmul(a, aOne, aInv, aScale, D, 1, 1)
        vec("mul", xt, aScale, aTmp + t * D, D)
        vec("mul", aTmp + t * D, aW, aOut + t * D, D)
    a.halt()
    return a.words, g.image(g.top), aOut, g.top


def swiglu_program(G: np.ndarray, U: np.ndarray):
    """silu(g) * u by the exp/add/div/mul recipe of test_swiglu.py:30-38 and
    legalize.py:130-149, over flat vectors (chunked)."""
    n = G.size
    g = GBuf(4 * n + 16)
    aZ = g.alloc(n)
    aOne = g.alloc(n); g.put(aOne, np.ones(n))
    aG = g.alloc(n); g.put(aG, G)
    aU = g.alloc(n); g.put(aU, U)
    aNg = g.alloc(n); aDen = g.alloc(n); aSig = g.alloc(n); aSilu = g.alloc(n); aH = g.alloc(n)
    a = Asm()
    ew(a, "sub", aNg, aZ, aG, n)
    ew(a, "exp", aDen, aNg, None, n)
    ew(a, "add", aDen, aDen, None, n, mode=IMM, imm=1)
    ew(a, "div", aSig, aOne, aDen, n)
    ew(a, "mul", aSilu, aG, aSig, n)
    ew(a, "mul", aH, aSilu, aU, n)
    a.halt()
    return a.words, g.image(g.top), aH, g.top


def softmax_program(S: np.ndarray, causal: bool = True):
    """Masked softmax rows by the reference recipe (test_attention.py:47-52,
    legalize.py:97-114): s + mask(-30000) -> exp -> rowsum (ones matmul) ->
    broadcast (ones matmul) -> divide.  No max subtraction.  [R, C], C <= 255."""
    R, C = S.shape
    g = GBuf()
    aS = g.alloc(R * C); g.put(aS, S)
    aMask = g.alloc(R * C)
    mask = np.where(np.arange(C)[None, :] <= np.arange(R)[:, None], 0.0, -30000.0) if causal else np.zeros((R, C))
    g.put(aMask, mask)
    aOne = g.alloc(C); g.put(aOne, np.ones(C))
    aE = g.alloc(R * C); aSum = g.alloc(R); aSB = g.alloc(R * C); aP = g.alloc(R * C)
    a = Asm()
    ew(a, "add", aS, aS, aMask, R * C)
    ew(a, "exp", aE, aS, None, R * C)
    matmul(a, aE, aOne, aSum, R, C, 1)
    matmul(a, aSum, aOne, aSB, R, 1, C)
    ew(a, "div", aP, aE, aSB, R * C)
    a.halt()
    return a.words, g.image(g.top), aP, g.top


def rope_program(Q: np.ndarray, cos: np.ndarray, sin: np.ndarray):
    """rope_Q macro of llama_layer.py:96-104: rh = [-q[h:], q[:h]] per token,
    then q*cos + rh*sin with fp16 tables.  Q [SEQ, HD]."""
    S, HD = Q.shape
    half = HD // 2
    g = GBuf()
    aQ = g.alloc(S * HD); g.put(aQ, Q)
    aC = g.alloc(S * HD); g.put(aC, cos)
    aS = g.alloc(S * HD); g.put(aS, sin)
    aZ = g.alloc(S * HD)
    aRh = g.alloc(S * HD); aT = g.alloc(S * HD); aO = g.alloc(S * HD)
    a = Asm()
    for t in range(S):
        base = aQ + t * HD
        ew(a, "sub", aRh + t * HD, aZ, base + half, half)
        ew(a, "add", aRh + t * HD + half, base, None, half, mode=IMM, imm=0)
    ew(a, "mul", aT, aQ, aC, S * HD)
    ew(a, "mul", aO, aRh, aS, S * HD)
    ew(a, "add", aO, aT, aO, S * HD)
    a.halt()
    return a.words, g.image(g.top), aO, g.top

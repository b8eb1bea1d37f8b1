"""Runners for the NPU cmodel -- TEST INFRASTRUCTURE ONLY (the checker).

Two executors of NPU programs:
  * `Machine` -- ctypes front-end of libisa_oracle.so, our C restatement of
    `_poc/mysim.cpp` (fp16 rounding :19-38, execute loop :83-145, stdout trace
    :69-75/87-88/100-104/142-144, write-back :147-155);
  * `run_mysim` -- the reference simulator itself, built from the reference's
    `_poc/mysim.cpp` into oracle/_ref/mysim by oracle/Makefile, driven exactly
    as the reference's `run()` drives it (b_program_examples/npu.py:62-71):
    files program_memory.bin / G_buffer_data.bin in a run directory,
    `mysim --run N --gout gout.bin --gn N`, fp16 write-back read back.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import tempfile
from typing import Optional, Sequence, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libisa_oracle.so")
MYSIM = os.path.join(HERE, "_ref", "mysim")

_lib = None


def build() -> None:
    """Build libisa_oracle.so (and oracle/_ref/mysim when the reference tree is present)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        P, I64, I = ctypes.c_void_p, ctypes.c_long, ctypes.c_int
        L.ora_create.restype = P
        L.ora_create.argtypes = [P, I64, I64]
        L.ora_destroy.argtypes = [P]
        L.ora_exec.restype = I64
        L.ora_exec.argtypes = [P, P, I64, I64, I, I64, I64]
        L.ora_error.restype = I
        L.ora_error.argtypes = [P]
        L.ora_trace_len.restype = I64
        L.ora_trace_len.argtypes = [P]
        L.ora_trace.restype = ctypes.c_void_p
        L.ora_trace.argtypes = [P]
        L.ora_gsize.restype = I64
        L.ora_gsize.argtypes = [P]
        L.ora_gread.argtypes = [P, P, I64]
        L.ora_f32_to_f16_array.argtypes = [P, P, I64]
        L.ora_vector.argtypes = [ctypes.c_uint32, P, P, P, P, I64]
        _lib = L
    return _lib


def f32_to_f16_bits(x) -> np.ndarray:
    """The cmodel's fp32 -> fp16 rounding (mysim.cpp:19-38) as uint16 bit patterns."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    y = np.empty(x.shape, dtype=np.uint16)
    lib().ora_f32_to_f16_array(x.ctypes.data, y.ctypes.data, x.size)
    return y


def vector_op(word: int, in1, in2=None, prev=None) -> np.ndarray:
    """fp32 result of one elementwise compute instruction (mysim.cpp:114-141)."""
    a = np.ascontiguousarray(np.asarray(in1, dtype=np.float32))
    b = None if in2 is None else np.ascontiguousarray(np.asarray(in2, dtype=np.float32))
    p = None if prev is None else np.ascontiguousarray(np.asarray(prev, dtype=np.float32))
    out = np.empty_like(a)
    lib().ora_vector(int(word) & 0xFFFFFFFF, a.ctypes.data, None if b is None else b.ctypes.data,
                     None if p is None else p.ctypes.data, out.ctypes.data, a.size)
    return out


def fp16_round(x) -> np.ndarray:
    """fp32 values rounded through the cmodel's fp16 store, back as fp32."""
    return f32_to_f16_bits(x).view(np.float16).astype(np.float32)


class Machine:
    """One cmodel instance over a G-buffer of fp16 words."""

    def __init__(self, gbuf_f16: np.ndarray, gcap: int = 1 << 16):
        g = np.ascontiguousarray(np.asarray(gbuf_f16).astype(np.float16).view(np.uint16))
        self._h = lib().ora_create(g.ctypes.data, g.size, max(gcap, g.size))
        if not self._h:
            raise MemoryError("ora_create failed")
        self.gin_n = g.size

    def close(self):
        if self._h:
            lib().ora_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def execute(self, words: Sequence[int], maxrun: int, trace: bool = False,
                gbytes: Optional[int] = None, pbytes: Optional[int] = None) -> Tuple[int, str]:
        """Run up to `maxrun` instructions; returns (steps, trace text or '')."""
        w = np.ascontiguousarray(np.asarray(words, dtype=np.uint32))
        gb = 2 * self.gin_n + 1 if gbytes is None else gbytes
        pb = 4 * w.size + 1 if pbytes is None else pbytes
        n = lib().ora_exec(self._h, w.ctypes.data, w.size, int(maxrun), 1 if trace else 0, gb, pb)
        if n < 0:
            raise RuntimeError(f"cmodel error {lib().ora_error(self._h)}")
        text = ""
        if trace:
            ln = lib().ora_trace_len(self._h)
            text = ctypes.string_at(lib().ora_trace(self._h), ln).decode()
        return int(n), text

    def gread(self, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.uint16)
        lib().ora_gread(self._h, out.ctypes.data, n)
        return out.view(np.float16)


def run_oracle(words: Sequence[int], gbuf: np.ndarray, gn: int, maxrun: int = 400) -> np.ndarray:
    """The C restatement run the way npu.run() runs mysim; returns G[0:gn] as fp16."""
    m = Machine(gbuf)
    try:
        m.execute(words, maxrun)
        return m.gread(gn)
    finally:
        m.close()


def have_mysim() -> bool:
    return os.path.exists(MYSIM) and os.access(MYSIM, os.X_OK)


def run_mysim(words: Sequence[int], gbuf: np.ndarray, gn: int, maxrun: int = 400,
              capture_trace: bool = False):
    """Run the reference simulator on (program, G-buffer) like npu.run(); returns
    G[0:gn] as fp16 (and the stdout trace when capture_trace)."""
    if not have_mysim():
        raise FileNotFoundError(f"{MYSIM} not built (make -C oracle with the reference tree present)")
    w = np.asarray(words, dtype="<u4")
    g = np.asarray(gbuf).astype("<f2")
    with tempfile.TemporaryDirectory() as d:
        with open(os.path.join(d, "program_memory.bin"), "wb") as f:
            f.write(w.tobytes() + b"\n")
        with open(os.path.join(d, "G_buffer_data.bin"), "wb") as f:
            f.write(g.tobytes() + b"\n")
        r = subprocess.run([MYSIM, "--run", str(maxrun), "--gout", os.path.join(d, "gout.bin"), "--gn", str(gn)],
                           cwd=d, check=True, stdout=subprocess.PIPE if capture_trace else subprocess.DEVNULL,
                           stderr=subprocess.DEVNULL)
        with open(os.path.join(d, "gout.bin"), "rb") as f:
            out = np.frombuffer(f.read()[: 2 * gn], dtype="<f2").copy()
    return (out, r.stdout.decode()) if capture_trace else out

"""Whole NPU programs on the GPU: the reference's run() entry points.

The reference builds programs (instruction words) with the macros of
b_program_examples/npu.py and the compiler of d_compiler/npu_compiler, and
executes them by writing program_memory.bin / G_buffer_data.bin and running
the cmodel in a subprocess:

    run(asm, gbuf, gn, rundir='.', maxrun=400)   b_program_examples/npu.py:62-71
    run(program, gbuf, gn=None, maxrun=None)     d_compiler/npu_compiler/runtime.py:46-77

Here the same calls execute the program on the GPU through the C ABI
(npub_program_create / _load / _run): the host decodes the straight-line
instruction stream into dependency-ordered tasks once, and one cooperative
kernel runs them with the cmodel's float32 semantics (its bits, except exp and
the matrix activation, which are within a few float32 ulps before the fp16
store).  A decoded Program can be run many times on different G-buffers.

Errors: a program that would read past a PE input buffer (undefined in the
cmodel) raises ValueError naming the program counter; CUDA failures raise
NpubError (the reference raises CalledProcessError when mysim fails).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np
import torch

from . import _lib, formats

__all__ = ["Program", "program_words", "run", "run_program"]


def program_words(program) -> np.ndarray:
    """Instruction words of a program given as the reference's Asm (`.p`), the
    compiler's Asm (`.words`), a program_memory.bin image (bytes) or a
    sequence of ints."""
    if isinstance(program, (bytes, bytearray, memoryview)):
        return formats.parse_program(bytes(program))
    for attr in ("p", "words"):
        if hasattr(program, attr):
            program = getattr(program, attr)
            break
    return np.asarray([int(w) & 0xFFFFFFFF for w in program], dtype=np.uint32)


def _gbuffer_words(gbuf, gn: Optional[int]) -> np.ndarray:
    """fp16 words of the initial G-buffer: the reference's GBuf writes its
    first gn entries (GBuf.bytes(gn), npu.py:58-60); arrays are taken whole."""
    if hasattr(gbuf, "bytes") and callable(gbuf.bytes):
        return formats.parse_gbuffer(gbuf.bytes(gn))
    if hasattr(gbuf, "image") and callable(gbuf.image):
        return np.asarray(gbuf.image(gn), dtype=np.float16)
    if hasattr(gbuf, "mem"):
        gbuf = gbuf.mem[:gn]
    if isinstance(gbuf, torch.Tensor):
        return gbuf.detach().to("cpu", torch.float16).numpy()
    return np.asarray(gbuf, dtype=np.float64).astype(np.float16)


class Program:
    """A decoded NPU program (npub_program_create) with its device workspace."""

    def __init__(self, program, maxrun: Optional[int] = None, g_in: int = 0, device=None):
        self.words = program_words(program)
        self.maxrun = len(self.words) + 1 if maxrun is None else int(maxrun)
        self.g_in = int(g_in)
        lib = _lib.load()
        h = ctypes.c_void_p()
        w = np.ascontiguousarray(self.words)
        st = lib.npub_program_create(w.ctypes.data if w.size else None, w.size, self.maxrun, self.g_in,
                                     ctypes.byref(h))
        if st != _lib.NPUB_OK:
            pc = lib.npub_program_error_pc()
            text = lib.npub_strerror(st).decode()
            if st == _lib.NPUB_ERR_INVALID_ARG:
                raise ValueError(f"program rejected at pc {pc}: an instruction reads past a PE input buffer "
                                 f"({text})")
            raise _lib.NpubError("npub_program_create", st, text)
        self._h = h
        info = (ctypes.c_int64 * 7)()
        lib.npub_program_info(h, info, 7)
        self.executed, self.tasks, self.levels, self.gwords, self.twords, self.chunks, self.ctas = list(info)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self._ws = None
        self._ws_bytes = 0

    def _workspace(self):
        if self._ws is None:
            lib = _lib.load()
            nb = int(lib.npub_program_workspace(self._h))
            raw = torch.empty(nb + 256, dtype=torch.uint8, device=self.device)
            off = (-raw.data_ptr()) % 256
            self._raw = raw
            self._ws = raw[off:off + nb]
            self._ws_bytes = nb
            _lib.call("npub_program_load", self._h, self._ws.data_ptr(), nb,
                      torch.cuda.current_stream(self.device).cuda_stream)
        return self._ws

    def run(self, g: torch.Tensor, gn: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Execute on the fp16 G-buffer g (CUDA, 1-D, at most the g_in words given
        at decode) and return the first gn words of the final G-buffer (fp16, CUDA)."""
        if not (isinstance(g, torch.Tensor) and g.is_cuda and g.dtype == torch.float16 and g.dim() == 1
                and g.is_contiguous()):
            raise ValueError("g must be a contiguous 1-D fp16 CUDA tensor")
        if g.numel() > self.g_in:
            raise ValueError(f"the G-buffer has {g.numel()} words, the program was decoded for {self.g_in}")
        ws = self._workspace()
        if out is None:
            out = torch.empty(gn, dtype=torch.float16, device=g.device)
        _lib.call("npub_program_run", self._h, g.data_ptr() if g.numel() else None, g.numel(),
                  out.data_ptr() if gn else None, int(gn), ws.data_ptr(), self._ws_bytes,
                  torch.cuda.current_stream(g.device).cuda_stream)
        return out

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.load().npub_program_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _execute(program, g16: np.ndarray, gn: int, maxrun: Optional[int]) -> np.ndarray:
    p = Program(program, maxrun=maxrun, g_in=g16.size)
    g = torch.from_numpy(np.ascontiguousarray(g16)).to(p.device)
    out = p.run(g, gn)
    res = out.cpu().numpy()
    p.close()
    return res


def run(asm, gbuf, gn: int, rundir: str = ".", maxrun: int = 400):
    """Run a program on the GPU like the reference's run() (npu.py:62-71): the
    initial G-buffer is gbuf's first gn entries rounded to fp16, at most maxrun
    instructions execute, and the first gn words of the final G-buffer come
    back as a list of floats.  `rundir` is accepted for the same signature; no
    files are written."""
    return [float(v) for v in _execute(asm, _gbuffer_words(gbuf, gn), int(gn), int(maxrun))]


def run_program(program, gbuf, gn: Optional[int] = None, maxrun: Optional[int] = None) -> np.ndarray:
    """The compiler runtime's run() (runtime.py:46-77): the whole gbuf is the
    initial G-buffer, gn defaults to its length and maxrun to the program length
    + 1; returns the written-back G-buffer as np.float32 [gn]."""
    g16 = _gbuffer_words(gbuf, None)
    gn = g16.size if gn is None else int(gn)
    return _execute(program, g16, gn, maxrun).astype(np.float32)

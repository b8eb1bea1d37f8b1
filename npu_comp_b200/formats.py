"""On-disk formats of the NPU toolchain, for interop and stage chaining.

  program_memory.bin   the program: 32-bit instruction words, little endian,
                       then one newline byte (b_program_examples/npu.py:39-40,
                       d_compiler/npu_compiler/isa.py:146-148).  A reader takes
                       the first filesize // 4 words and ignores the rest, as
                       the cmodel does (_poc/mysim.cpp:60-66) and
                       read_program_bin (isa.py:193-199).
  G_buffer_data.bin    the G-buffer: IEEE binary16 words, little endian, then
                       one newline byte (npu.py:58-60, runtime.py:40-43); the
                       cmodel reads filesize // 2 words (mysim.cpp:51-56).
  gout.bin             the cmodel's --gout write-back, the same format as
                       G_buffer_data.bin (mysim.cpp:147-155): the first gn words
                       of the final G-buffer, so one program's output can be the
                       next program's input.
"""
from __future__ import annotations

import os
from typing import Iterable, Sequence, Union

import numpy as np

PROGRAM_FILE = "program_memory.bin"
GBUFFER_FILE = "G_buffer_data.bin"


def program_bytes(words: Iterable[int]) -> bytes:
    """Words -> the program_memory.bin image (uint32 LE + newline)."""
    w = np.asarray([int(x) & 0xFFFFFFFF for x in words], dtype="<u4")
    return w.tobytes() + b"\n"


def parse_program(data: bytes) -> np.ndarray:
    """program_memory.bin image -> uint32 words (a trailing partial word, the
    newline, is ignored)."""
    n = len(data) // 4
    return np.frombuffer(data[: 4 * n], dtype="<u4").astype(np.uint32)


def write_program_bin(path: str, words: Iterable[int]) -> None:
    with open(path, "wb") as f:
        f.write(program_bytes(words))


def read_program_bin(path: str) -> np.ndarray:
    with open(path, "rb") as f:
        return parse_program(f.read())


def gbuffer_bytes(values: Union[Sequence[float], np.ndarray]) -> bytes:
    """Values -> the G_buffer_data.bin image (each rounded to fp16, LE + newline)."""
    return np.asarray(values, dtype=np.float64).astype("<f2").tobytes() + b"\n"


def parse_gbuffer(data: bytes) -> np.ndarray:
    """G_buffer_data.bin / gout.bin image -> fp16 words (the trailing byte ignored)."""
    n = len(data) // 2
    return np.frombuffer(data[: 2 * n], dtype="<f2").astype(np.float16)


def write_gbuffer_bin(path: str, values) -> None:
    with open(path, "wb") as f:
        f.write(gbuffer_bytes(values))


def read_gbuffer_bin(path: str) -> np.ndarray:
    with open(path, "rb") as f:
        return parse_gbuffer(f.read())


def read_rundir(rundir: str):
    """(program words, G-buffer words) from the two input files of a run directory."""
    return (read_program_bin(os.path.join(rundir, PROGRAM_FILE)),
            read_gbuffer_bin(os.path.join(rundir, GBUFFER_FILE)))

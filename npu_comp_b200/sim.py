"""Command-line stand-in for the cmodel binary, executing on the GPU.

    python -m npu_comp_b200.sim [--run N] [--gout FILE] [--gn N] [--gbuf CAP]

reads program_memory.bin and G_buffer_data.bin from the current directory and
writes the first gn words of the final G-buffer to FILE, with the arguments
and file formats of _poc/mysim.cpp:42-66,147-155 (defaults: --run 30, gn =
the input's word count).  A run directory prepared for the reference's run()
(b_program_examples/npu.py:62-71) can therefore be executed here unchanged.
The per-instruction stdout trace of the cmodel is not produced; a summary
line goes to stderr.
"""
from __future__ import annotations

import argparse
import os
import sys


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--run", type=int, default=30, help="maximum program-counter steps")
    ap.add_argument("--gout", default=None, help="write-back file (fp16 LE + newline)")
    ap.add_argument("--gn", type=int, default=-1, help="words to write back (default: the input's)")
    ap.add_argument("--gbuf", type=int, default=1 << 16, help="initial G-buffer capacity (accepted; it grows)")
    a = ap.parse_args(argv)
    import torch
    from . import formats
    from .program import Program
    words, g16 = formats.read_rundir(os.getcwd())
    prog = Program(words, maxrun=a.run, g_in=g16.size)
    gn = g16.size if a.gn < 0 else a.gn
    out = prog.run(torch.from_numpy(g16.copy()).to(prog.device), gn)
    if a.gout:
        formats.write_gbuffer_bin(a.gout, out.float().cpu().numpy())
    sys.stderr.write(f"[npu_comp_b200.sim] {prog.executed} steps, {prog.tasks} tasks in {prog.levels} levels; "
                     f"wrote {gn if a.gout else 0} FP16 entries" + (f" -> {a.gout}\n" if a.gout else "\n"))
    prog.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())

"""NPU programs for the program-executor tests: the reference's own captured
programs (tests/golden/programs.npz), the ISA golden programs and seeded
random programs, with a helper comparing fp16 G-buffer images.

Random programs are built from the reference's instruction forms
(b_program_examples/npu.py:10-47, _poc/README.md:84-114) and are valid by
construction: every compute reads no more than its loads provided."""
import json
import os

import numpy as np

from oracle import emit

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
EXP_OPS = (0x0F,)


def captured_programs():
    """[(name, words, gin fp16, gn, maxrun, gout fp16)] of the example scripts' run() calls."""
    d = np.load(os.path.join(GOLDEN, "programs.npz"))
    names = sorted({k.rsplit("_", 1)[0] for k in d.files})
    return [(n, d[n + "_words"], d[n + "_gin"], int(d[n + "_gn"]), int(d[n + "_maxrun"]), d[n + "_gout"])
            for n in names]


def isa_programs():
    with open(os.path.join(GOLDEN, "isa_goldens.json")) as f:
        g = json.load(f)
    out = []
    for p in g["programs"]:
        w = np.zeros(p["nwords"], dtype=np.uint32)
        w[: len(p["words"])] = p["words"]
        out.append((p["name"], w, g["maxrun"]))
    return out


def ramp():
    return np.arange(8192).astype(np.float16)


def uses_exp(words) -> bool:
    """Whether a program has exp or an activated matrix op (CUDA expf vs libm)."""
    for w in np.asarray(words, dtype=np.uint32):
        op = int(w) & 0xFF
        if op == 0x0F or (0x40 <= op <= 0x43 and (int(w) >> 29) & 1):
            return True
    return False


def ulp_diff(a16, b16) -> np.ndarray:
    """Distance in fp16 ulps between two fp16 arrays (NaN == NaN, -0 == +0)."""
    a = np.asarray(a16, np.float16).view(np.uint16).astype(np.int32)
    b = np.asarray(b16, np.float16).view(np.uint16).astype(np.int32)

    def key(u):  # monotone integer line: negative values below positive ones
        return np.where(u & 0x8000, -(u & 0x7FFF), u & 0x7FFF)
    na, nb = np.isnan(np.asarray(a16, np.float16)), np.isnan(np.asarray(b16, np.float16))
    d = np.abs(key(a) - key(b))
    d[na & nb] = 0
    d[na ^ nb] = 1 << 20
    return d


def random_gbuffer(rng, n=12000):
    """Mixed values: small integers (logic, shift, convert), normals, large values, a few inf / nan."""
    g = rng.standard_normal(n) * 4
    k = rng.random(n)
    g = np.where(k < 0.3, np.round(rng.uniform(-300, 300, n)), g)
    g = np.where((k > 0.95) & (k < 0.97), rng.uniform(-6e4, 6e4, n), g)
    g[rng.integers(0, n, 20)] = np.inf
    g[rng.integers(0, n, 20)] = -np.inf
    g[rng.integers(0, n, 10)] = np.nan
    return g.astype(np.float16)


ELEM_OPS = [0x01, 0x02, 0x0A, 0x0B, 0x0C, 0x0D, 0x0E, 0x11, 0x12, 0x13, 0x09, 0x08]


def random_program(rng, n_groups=60, with_exp=False, gsize=12000):
    """A random, valid program (list of words) over a G-buffer of gsize words."""
    a = emit.Asm()
    ops = ELEM_OPS + ([0x0F] if with_exp else [])
    loaded = [0, 0]
    for _ in range(n_groups):
        kind = rng.random()
        if kind < 0.6:  # elementwise group: vlen, loads, compute(s), saves
            n = int(rng.integers(1, 400))
            a.vlen(n)
            a.addr(emit.SRC1, int(rng.integers(0, gsize - n)))
            a.load(0, 0)
            loaded[0] = n
            if rng.random() < 0.8:
                a.addr(emit.SRC2, int(rng.integers(0, gsize - n)))
                a.load(0, 1)
                loaded[1] = n
            if rng.random() < 0.15:  # a save over the loaded range before the compute reads it
                a.addr(emit.DST, int(rng.integers(0, gsize - n)))
                a.save(0)
            for _ in range(int(rng.integers(1, 3))):  # chained computes: mul-add reads the previous output
                op = int(rng.choice(ops))
                mode = int(rng.choice([0, 1, 2] if loaded[1] >= n else [0, 1]))
                imm = int(rng.integers(0, 1 << 16)) if op != 0x09 else int(rng.integers(-40, 40)) & 0xFFFF
                sub = int(rng.integers(0, 6)) if op == 0x08 else 0
                bit28 = int(rng.integers(0, 2)) if op == 0x12 else 0
                a.compute({v: k for k, v in emit.OP.items()}[op], mode, imm, bit28=bit28, sub=sub)
            # now and then far past the initial 65536-word buffer, which then grows
            far = rng.random() < 0.05
            a.addr(emit.DST, int(rng.integers(70000, 80000)) if far else int(rng.integers(0, gsize - n)))
            a.save(0)
        elif kind < 0.85:  # matrix multiply (optionally activated)
            rA, cA, cB = (int(rng.integers(1, 40)) for _ in range(3))
            a.tile(0, rA, cA)
            a.tile(1, cA, cB)
            a.addr(emit.SRC1, int(rng.integers(0, gsize - rA * cA)))
            a.addr(emit.SRC2, int(rng.integers(0, gsize - cA * cB)))
            a.load(1, 0)
            a.load(1, 1)
            loaded = [rA * cA, cA * cB]
            a.m_mul(mode=emit.VECTOR, act=with_exp and rng.random() < 0.5)
            a.addr(emit.DST, int(rng.integers(0, gsize - rA * cB)))
            a.save(1)
        else:  # matrix elementwise op over tA[0] x tB[0]
            r, c = int(rng.integers(1, 20)), int(rng.integers(1, 20))
            a.tile(0, r, c)
            a.tile(1, r, c)
            a.addr(emit.SRC1, int(rng.integers(0, gsize - r * c)))
            a.addr(emit.SRC2, int(rng.integers(0, gsize - r * c)))
            a.load(1, 0)
            a.load(1, 1)
            loaded = [r * c, r * c]
            op = int(rng.choice([0x40, 0x41, 0x42, 0x43]))
            mode = int(rng.choice([0, 2])) if op != 0x42 else 0
            a.compute({v: k for k, v in emit.OP.items()}[op], mode, int(rng.integers(0, 100)),
                      act=with_exp and rng.random() < 0.5)
            a.addr(emit.DST, int(rng.integers(0, gsize - r * c)))
            a.save(1)
        if rng.random() < 0.05:
            a.nop()
    a.halt()
    return a.words

"""Host side of the program executor and the on-disk formats (CPU).

* The captured programs of the reference's example scripts (tests/golden/
  programs.npz, made by tests/golden/make_goldens.py from the scripts' own
  run() calls): the C restatement of the cmodel reproduces each write-back
  word for word, which pins the fixtures the GPU tests compare with.
* npub_program_create decodes on the host (no GPU needed): dependency levels,
  steps, the rejection of programs that read past a PE buffer.
* program_memory.bin / G_buffer_data.bin round trips (formats.py).
"""
import ctypes

import numpy as np
import pytest

from npu_comp_b200 import _lib, formats
from oracle import cmodel, emit
from tests import program_cases as pc


@pytest.mark.parametrize("case", pc.captured_programs(), ids=lambda c: c[0])
def test_captured_program_oracle_reproduces_simulator(case):
    name, words, gin, gn, maxrun, gout = case
    got = cmodel.run_oracle(words, gin, gn, maxrun=maxrun)
    assert np.array_equal(got.view(np.uint16), gout.view(np.uint16)), name


def _create(words, maxrun, g_in):
    lib = _lib.load()
    h = ctypes.c_void_p()
    w = np.ascontiguousarray(np.asarray(words, dtype=np.uint32))
    st = lib.npub_program_create(w.ctypes.data if w.size else None, w.size, maxrun, g_in, ctypes.byref(h))
    info = (ctypes.c_int64 * 7)()
    if st == 0:
        lib.npub_program_info(h, info, 7)
    return st, h, list(info)


def test_decode_levels_and_steps(libnpub_path):
    lib = _lib.load()
    for name, words, gin, gn, maxrun, gout in pc.captured_programs():
        st, h, info = _create(words, maxrun, gin.size)
        assert st == 0, name
        steps, tasks, levels, gwords, twords, chunks, ctas = info
        nz = int(np.nonzero(words == 0xFF)[0][0]) + 1 if (words == 0xFF).any() else len(words)
        assert steps == min(nz, maxrun)
        assert 0 < levels <= tasks
        assert gwords >= max(65536, gin.size)
        assert lib.npub_program_workspace(h) >= (gwords + twords) * 4
        lib.npub_program_destroy(h)
    # the 71,017-instruction 64-tiled matmul program of the single W8A16 configuration
    rng = np.random.default_rng(0)
    A = rng.standard_normal((64, 512)).astype(np.float16)
    Wd = (rng.standard_normal((512, 512)) * 0.02).astype(np.float16)
    words, gimg, _, _ = emit.w8a16_program(A, Wd)
    st, h, info = _create(words, len(words) + 1, len(gimg))
    assert st == 0 and info[0] == len(words)
    assert info[2] < 200        # ~17.6 K tasks in ~130 dependency levels
    lib.npub_program_destroy(h)


def test_decode_rejects_reads_past_a_pe_buffer(libnpub_path):
    a = emit.Asm()
    a.vlen(8)
    a.addr(emit.SRC1, 0)
    a.load(0, 0)
    a.vlen(16)               # the compute wants 16 elements, the load gave 8
    a.v_add(mode=emit.IMM, imm=1)
    a.halt()
    st, h, _ = _create(a.words, 100, 64)
    assert st == _lib.NPUB_ERR_INVALID_ARG
    assert _lib.load().npub_program_error_pc() == 5   # vlen, addr (2 words), load, vlen, add
    # maxrun ends the program before the faulty instruction: accepted
    st, h, info = _create(a.words, 5, 64)
    assert st == 0 and info[0] == 5
    _lib.load().npub_program_destroy(h)


def test_program_file_round_trip(tmp_path):
    words = [0, 0x80, 0xFF, 0xDEADBEEF, 12345]
    p = tmp_path / "program_memory.bin"
    formats.write_program_bin(str(p), words)
    raw = p.read_bytes()
    assert len(raw) == 4 * len(words) + 1 and raw[-1:] == b"\n"
    assert formats.read_program_bin(str(p)).tolist() == words


def test_gbuffer_file_round_trip(tmp_path):
    v = np.array([0.0, -0.0, 1.5, 65504.0, 1e-7, np.inf, -np.inf], dtype=np.float64)
    p = tmp_path / "G_buffer_data.bin"
    formats.write_gbuffer_bin(str(p), v)
    raw = p.read_bytes()
    assert len(raw) == 2 * v.size + 1 and raw[-1:] == b"\n"
    got = formats.read_gbuffer_bin(str(p))
    assert np.array_equal(got.view(np.uint16), v.astype(np.float16).view(np.uint16))


def test_random_programs_are_valid_for_the_oracle():
    rng = np.random.default_rng(3)
    g = pc.random_gbuffer(rng)
    for _ in range(3):
        words = pc.random_program(rng)
        m = cmodel.Machine(g)
        m.execute(words, len(words) + 1)   # raises on a machine error
        m.close()


def test_oracle_nan_rules_equal_reference_simulator():
    """The C restatement's NaN results (SSE: quiet NaN operands propagate, the
    destination-register operand winning when both are NaN; invalid operations
    give the negative indefinite NaN) equal the reference simulator's on
    random programs over G-buffers with inf, nan and integers."""
    if not cmodel.have_mysim():
        pytest.skip("reference simulator not built here")
    for seed in range(8):
        rng = np.random.default_rng(1000 + seed)
        g = pc.random_gbuffer(rng)
        words = pc.random_program(rng, n_groups=60, with_exp=seed % 2 == 0)
        o = cmodel.run_oracle(words, g, 80000, maxrun=len(words) + 1)
        m = cmodel.run_mysim(words, g, 80000, maxrun=len(words) + 1)
        assert np.array_equal(o.view(np.uint16), m.view(np.uint16)), seed

"""Whole NPU programs on the GPU (npu_comp_b200.program: the reference's run()
entry points on npub_program_*) against the cmodel.

* The programs the reference's example scripts hand to run() (test_matmul,
  test_rmsnorm, test_swiglu, test_attention and the full llama_layer.py
  program, captured with their G-buffers in tests/golden/programs.npz), the
  55 ISA golden programs on the ramp G-buffer, the 71,017-instruction
  64-tiled W8A16 matmul of the single-matmul configuration, and seeded
  random programs (every opcode, integer-valued ops on integers, inf / nan,
  mul-add chains, saves over loaded ranges, buffer growth).
* Bit-exact: the final G-buffer equals the cmodel's word for word, except for
  programs with exp or an activated matrix op, where CUDA's expf may move a
  word by one fp16 ulp (and the normwise relative error stays within TOL).
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from npu_comp_b200 import formats, program
from oracle import cmodel, emit, ref
from tests import program_cases as pc

pytestmark = pytest.mark.gpu
TOL = 1e-2
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def gpu_run(words, gin, gn, maxrun):
    p = program.Program(words, maxrun=maxrun, g_in=len(gin))
    out = p.run(torch.from_numpy(np.ascontiguousarray(gin)).cuda(), gn).cpu().numpy()
    info = (p.tasks, p.levels)
    p.close()
    return out, info


def check(name, got, want, words):
    if pc.uses_exp(words):
        d = pc.ulp_diff(got, want)
        assert d.max() <= 1, (name, int(d.max()), int((d > 0).sum()))
        fin = np.isfinite(want.astype(np.float32))
        assert ref.rel_err(got.astype(np.float32)[fin], want.astype(np.float32)[fin]) <= TOL
    else:
        assert np.array_equal(got.view(np.uint16), want.view(np.uint16)), \
            (name, int((got.view(np.uint16) != want.view(np.uint16)).sum()))


@pytest.mark.parametrize("case", pc.captured_programs(), ids=lambda c: c[0])
def test_reference_example_programs(cuda_device, case):
    name, words, gin, gn, maxrun, gout = case
    got, (tasks, levels) = gpu_run(words, gin, gn, maxrun)
    check(name, got, gout, words)


def test_reference_llama_layer_program_through_run_api(cuda_device):
    """The llama_layer.py program through run() with the reference's signature:
    the G-buffer object's bytes(gn) image is what the machine starts from."""
    name, words, gin, gn, maxrun, gout = [c for c in pc.captured_programs() if c[0].startswith("llama_layer")][0]

    class Asm:  # the reference's Asm keeps its words in .p (npu.py:10-13)
        p = [int(w) for w in words]

    class GBuf:  # and its G-buffer writes bytes(count) (npu.py:49-60)
        def __init__(self, g):
            self.g = g

        def bytes(self, count):
            return formats.gbuffer_bytes(self.g[:count].astype(np.float64))

    out = program.run(Asm(), GBuf(gin), gn, rundir=".", maxrun=maxrun)
    assert isinstance(out, list) and len(out) == gn
    check(name, np.asarray(out, np.float64).astype(np.float16), gout, words)


@pytest.mark.parametrize("case", pc.isa_programs(), ids=lambda c: c[0])
def test_isa_golden_programs(cuda_device, case):
    name, words, maxrun = case
    g = pc.ramp()
    want = cmodel.run_oracle(words, g, 65536, maxrun=maxrun)
    got, _ = gpu_run(words, g, 65536, maxrun)
    check(name, got, want, words)


def test_tiled_w8a16_program_equals_reference_simulator(cuda_device):
    """The 64-tiled program of the single W8A16 configuration (64 x 512 x 512,
    71,017 instructions, codegen.py:59-108) against the reference simulator's
    output recorded in tests/golden/w8a16_config1.npz."""
    fx = np.load(os.path.join(ROOT, "tests", "golden", "w8a16_config1.npz"))
    rng = np.random.default_rng(0)
    A = rng.standard_normal((64, 512)).astype(np.float16)
    W = (rng.standard_normal((512, 512)) * 0.02).astype(np.float32)
    q, s = ref.quantize_w8(W)
    words, gimg, ca, gn = emit.w8a16_program(A, ref.dequant_f16(q, s))
    assert len(words) == int(fx["instructions"])
    got, (tasks, levels) = gpu_run(words, gimg, gn, len(words) + 1)
    C = got[ca: ca + 64 * 512].reshape(64, 512)
    assert np.array_equal(C.view(np.uint16), fx["C_mysim"].view(np.uint16))
    assert levels < 200


def cmodel_run(words, g, gn):
    """The reference simulator's write-back when it is built here, else the C restatement's."""
    if cmodel.have_mysim():
        return cmodel.run_mysim(words, g, gn, maxrun=len(words) + 1)
    return cmodel.run_oracle(words, g, gn, maxrun=len(words) + 1)


@pytest.mark.parametrize("seed", range(6))
def test_random_programs_bit_exact(cuda_device, seed):
    """inf / nan / integer-valued G-buffers: NaN signs (SSE rules) included."""
    rng = np.random.default_rng(100 + seed)
    g = pc.random_gbuffer(rng)
    words = pc.random_program(rng, n_groups=80)
    want = cmodel_run(words, g, 80000)
    got, _ = gpu_run(words, g, 80000, len(words) + 1)
    check(f"random{seed}", got, want, words)


@pytest.mark.parametrize("seed", range(4))
def test_random_programs_with_exp_and_activation(cuda_device, seed):
    rng = np.random.default_rng(200 + seed)
    g = (rng.standard_normal(12000) * 2).astype(np.float16) if seed < 2 else pc.random_gbuffer(rng)
    words = pc.random_program(rng, n_groups=60, with_exp=True)
    want = cmodel_run(words, g, 80000)
    got, _ = gpu_run(words, g, 80000, len(words) + 1)
    check(f"random_exp{seed}", got, want, words)


def test_program_reruns_and_run_program_api(cuda_device):
    """One decoded program runs on several G-buffers; the compiler runtime's
    run_program() (runtime.py:46-77) returns float32 of the whole buffer."""
    rng = np.random.default_rng(7)
    words = pc.random_program(rng, n_groups=30)
    p = program.Program(words, g_in=12000)
    for k in range(3):
        g = pc.random_gbuffer(np.random.default_rng(k))
        got = p.run(torch.from_numpy(g).cuda(), 12000).cpu().numpy()
        want = cmodel_run(words, g, 12000)
        assert np.array_equal(got.view(np.uint16), want.view(np.uint16))
    p.close()
    g = pc.random_gbuffer(np.random.default_rng(9))
    out = program.run_program(np.asarray(words, np.uint32), g.astype(np.float32))
    assert out.dtype == np.float32 and out.shape == (12000,)
    want = cmodel_run(words, g, 12000).astype(np.float32)
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32))


def test_cli_in_a_run_directory(cuda_device, tmp_path):
    """python -m npu_comp_b200.sim in a directory holding program_memory.bin and
    G_buffer_data.bin writes gout.bin like the cmodel's --gout."""
    name, words, gin, gn, maxrun, gout = pc.captured_programs()[0]
    formats.write_program_bin(str(tmp_path / formats.PROGRAM_FILE), words)
    formats.write_gbuffer_bin(str(tmp_path / formats.GBUFFER_FILE), gin.astype(np.float64))
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run([sys.executable, "-m", "npu_comp_b200.sim", "--run", str(maxrun), "--gout",
                        str(tmp_path / "gout.bin"), "--gn", str(gn)], cwd=tmp_path, env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    got = formats.read_gbuffer_bin(str(tmp_path / "gout.bin"))
    assert (tmp_path / "gout.bin").read_bytes()[-1:] == b"\n"
    check(name, got, gout, words)

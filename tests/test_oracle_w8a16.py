"""W8A16 oracle (CPU).  The reference has no int8 path; its matmul is the
64-tiled fp16 program of d_compiler/npu_compiler/codegen.py:59-108 run on
mysim.  The W8A16 oracle dequantises on the host (fp16(q*s)) and runs that
program; the quantiser itself is pinned by known-answer cases."""
import hashlib
import os

import numpy as np

from oracle import cmodel, emit, ref

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def config1_inputs():
    rng = np.random.default_rng(0)
    A = rng.standard_normal((64, 512)).astype(np.float16)
    W = (rng.standard_normal((512, 512)) * 0.02).astype(np.float32)
    return A, W


def test_config1_inputs_are_the_fixture_inputs():
    A, W = config1_inputs()
    g = np.load(os.path.join(GOLDEN, "w8a16_config1.npz"))
    assert hashlib.sha256(A.tobytes()).hexdigest() == str(g["sha_A"])
    assert hashlib.sha256(W.tobytes()).hexdigest() == str(g["sha_W"])


def test_config1_program_on_c_oracle_matches_reference_simulator():
    A, W = config1_inputs()
    q, s = ref.quantize_w8(W)
    words, gimg, ca, gn = emit.w8a16_program(A, ref.dequant_f16(q, s))
    g = np.load(os.path.join(GOLDEN, "w8a16_config1.npz"))
    assert len(words) == int(g["instructions"]) == 71017  # codegen.py tiling of 64x512x512
    C = cmodel.run_oracle(words, gimg, gn, maxrun=len(words) + 1)[ca: ca + 64 * 512].reshape(64, 512)
    assert np.array_equal(C.view(np.uint16), g["C_mysim"].view(np.uint16))
    # tiled_fp16_ref (d_compiler/tests/test_tiling.py:37-47) is byte-exact with the program
    assert np.array_equal(C.astype(np.float32), ref.tiled_fp16_ref(A, ref.dequant_f16(q, s)))
    # and within the fp16 tolerance of the exact W8A16 product
    assert ref.rel_err(C, ref.w8a16_ref(A, q, s)) < 1e-2


def test_quantizer_known_answers():
    # power-of-two column maxima give exact scales and exact integer codes
    W = np.zeros((4, 3), np.float32)
    W[:, 0] = [127 * 2.0 ** -8, -1 * 2.0 ** -8, 0.0, 64 * 2.0 ** -8]
    W[:, 1] = [-127 * 2.0 ** -4, 127 * 2.0 ** -4, 3 * 2.0 ** -4, -5 * 2.0 ** -4]
    W[:, 2] = 0.0  # an all-zero column: scale 0, codes 0
    q, s = ref.quantize_w8(W)
    assert q.shape == (3, 4) and q.dtype == np.int8 and s.dtype == np.float16
    assert s[0] == np.float16(2.0 ** -8) and s[1] == np.float16(2.0 ** -4) and s[2] == 0
    assert q[0].tolist() == [127, -1, 0, 64]
    assert q[1].tolist() == [-127, 127, 3, -5]
    assert q[2].tolist() == [0, 0, 0, 0]


def test_quantizer_extremes_and_k1(rng):
    W = (rng.standard_normal((1, 33)) * 0.3).astype(np.float32)  # K = 1: every code is +-127
    q, s = ref.quantize_w8(W)
    assert np.all(np.abs(q[:, 0]) == 127)
    W = (rng.standard_normal((300, 50)) * 0.02).astype(np.float32)
    q, s = ref.quantize_w8(W)
    assert np.abs(q).max() <= 127
    # each column reaches +-127 (the absmax element) unless fp16 rounding of the
    # scale pulls it to 126
    assert np.all(np.abs(q).max(axis=1) >= 126)
    # dequantisation error is at most half a step per element
    err = np.abs(q.T.astype(np.float64) * s.astype(np.float64) - W)
    assert np.all(err <= 0.5 * s.astype(np.float64)[None, :] * (1 + 1e-3) + 1e-12)


def test_w8a16_power_of_two_known_answer():
    # integer activations x power-of-two scales: every product and sum is exact
    A = np.array([[1, -2, 3, 0], [4, 5, -6, 7]], np.float16)
    q = np.array([[1, 2, 3, 4], [-5, 6, -7, 8], [127, -127, 0, 1]], np.int8)
    s = np.array([0.5, 0.25, 2.0 ** -6], np.float16)
    out = ref.w8a16_ref(A, q, s)
    assert np.array_equal(out, np.array([[3.0, -9.5, (127 + 254) * 2.0 ** -6],
                                         [12.0, 27.0, (508 - 635 + 7) * 2.0 ** -6]]))

"""Single-instruction semantics of the C restatement of the cmodel (CPU),
beyond the golden traces: out-of-range, NaN and signed cases of the integer-
valued ops, whose x86-64 behaviour (mysim.cpp:130-136, compiled with g++) the
GPU kernels must reproduce bit for bit."""
import numpy as np
import pytest

from oracle import cmodel, emit

INT64_MIN = -(2 ** 63)


def run_vec(word, a, b=None, prev=None):
    """Execute one vector compute instruction on PE buffers loaded from the G-buffer."""
    a = np.asarray(a, np.float16)
    n = a.size
    g = np.zeros(4 * n + 16, np.float16)
    g[:n] = a
    if b is not None:
        g[n:2 * n] = np.asarray(b, np.float16)
    if prev is not None:
        g[2 * n:3 * n] = np.asarray(prev, np.float16)
    asm = emit.Asm()
    asm.vlen(n)
    if prev is not None:  # previous PE output = prev (move), for mul-add
        asm.addr(emit.SRC2, 2 * n)
        asm.load(0, 1)
        asm.addr(emit.SRC1, 2 * n)
        asm.load(0, 0)
        asm.v_move(mode=emit.VECTOR)
    asm.addr(emit.SRC1, 0)
    asm.load(0, 0)
    if b is not None:
        asm.addr(emit.SRC2, n)
        asm.load(0, 1)
    asm.emit(word)
    asm.addr(emit.DST, 3 * n)
    asm.save(0)
    asm.halt()
    out = cmodel.run_oracle(asm.words, g, g.size, maxrun=len(asm.words) + 1)
    if cmodel.have_mysim():  # the reference simulator agrees bit for bit
        sim = cmodel.run_mysim(asm.words, g, g.size, maxrun=len(asm.words) + 1)
        assert np.array_equal(sim.view(np.uint16), out.view(np.uint16))
    return out[3 * n: 4 * n].astype(np.float32)


def test_convert_truncates_toward_zero():
    x = [1.5, -1.5, 2.75, -0.25, 65504.0, -65504.0, 1000.5]
    got = run_vec(0x13, x)
    assert got.tolist() == [1.0, -1.0, 2.0, 0.0, 65504.0, -65504.0, 1000.0]


def test_convert_inf_nan_give_int64_min():
    got = run_vec(0x13, [np.inf, -np.inf, np.nan])
    # (float)INT64_MIN = -2^63 -> fp16 store overflows to -inf
    assert np.all(np.isneginf(got))


@pytest.mark.parametrize("sub,fn", [(0, lambda a, b: a & b), (1, lambda a, b: a | b), (3, lambda a, b: a ^ b),
                                    (4, lambda a, b: ~(a & b)), (5, lambda a, b: ~(a | b))])
def test_logical_ops_on_long_casts(sub, fn):
    a = [5.0, -6.0, 7.9, -0.5, 100.0]
    b = [3.0, 3.0, -2.0, 9.0, 27.0]
    got = run_vec((2 << 30) | (sub << 27) | 0x08, a, b)
    exp = [np.float16(np.float32(fn(int(x), int(y)))) for x, y in zip(a, b)]
    assert got.tolist() == [float(e) for e in exp]


def test_logical_not_and_nan_operand():
    got = run_vec((0 << 30) | (2 << 27) | 0x08, [0.0, 5.0, -1.0, np.nan])
    assert got[:3].tolist() == [-1.0, -6.0, 0.0]
    # NaN -> INT64_MIN, ~INT64_MIN = INT64_MAX -> 2^63 in float -> +inf in fp16
    assert np.isposinf(got[3])


def test_shift_is_scaling_by_power_of_two():
    # shift amount from a vector operand; (int16)(int) conversion of large values wraps
    a = [1.0, 3.0, -2.0, 1.0, 1.0]
    b = [3.0, -1.0, 4.0, -30.0, 20.0]
    got = run_vec((2 << 30) | 0x09, a, b)
    assert got.tolist() == [8.0, 1.5, -32.0, np.float32(np.float16(2.0 ** -30)), np.inf]


def test_compare_min_max_nan_rules():
    a = [1.0, 2.0, np.nan, 3.0]
    b = [1.0, 3.0, 1.0, np.nan]
    assert run_vec((2 << 30) | 0x11, a, b).tolist() == [1.0, 0.0, 0.0, 0.0]
    mx = run_vec((2 << 30) | (1 << 28) | 0x12, a, b)
    # a > b ? a : b  -- NaN in a gives b, NaN in b gives b (NaN)
    assert mx[:3].tolist() == [1.0, 3.0, 1.0] and np.isnan(mx[3])


def test_muladd_uses_previous_output_two_roundings():
    got = run_vec((2 << 30) | 0x0C, [0.1, 3.0], [0.2, 4.0], prev=[1.0, -12.0])
    exp = np.float32(1.0) + np.float32(np.float16(0.1)) * np.float32(np.float16(0.2))
    assert got[0] == np.float32(np.float16(exp)) and got[1] == 0.0


def test_fp16_store_rounding_edges():
    x = np.array([65504.0, 65519.0, 65520.0, 2.0 ** -24, 2.0 ** -25, 2.0 ** -25 * 1.5, -0.0, np.nan, -np.nan],
                 np.float32)
    h = cmodel.f32_to_f16_bits(x)
    assert h[:7].tolist() == [0x7BFF, 0x7BFF, 0x7C00, 0x0001, 0x0000, 0x0001, 0x8000]
    assert h[7] == 0x7E00 and h[8] == 0xFE00

"""The NPU's elementwise instruction semantics on the GPU (npub_isa_vector)
against the C restatement of the cmodel, over every compute instruction word
the 55 golden ISA programs contain plus edge values.  Integer-valued ops
(logical, shift, compare, convert), min/max, move and IEEE add/sub/mul/div/
sqrt are bit-exact; exp and the x^2*sigmoid activation are within 4 float32
ulps."""
import json
import os

import numpy as np
import pytest
import torch

import npu_comp_b200 as nb
from oracle import cmodel

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def compute_words():
    with open(os.path.join(GOLDEN, "isa_goldens.json")) as f:
        progs = json.load(f)["programs"]
    words = set()
    for p in progs:
        for w in p["words"]:
            op = w & 0xFF
            if (0x01 <= op <= 0x13 or 0x40 <= op <= 0x43) and not (op == 0x42 and (w >> 30) & 3 == 2):
                words.add(w)
    return sorted(words)


WORDS = compute_words()
EXTRA = [(2 << 30) | (s << 27) | 0x08 for s in range(6)] + [0x13, (2 << 30) | 0x09, (2 << 30) | 0x11,
                                                            (2 << 30) | (1 << 28) | 0x12, (2 << 30) | 0x12]


def inputs(rng, n=4096):
    a = np.concatenate([np.arange(-64, 64, dtype=np.float32) * 0.75,
                        rng.standard_normal(n) * 30,
                        np.array([np.inf, -np.inf, np.nan, 0.0, -0.0, 65504, -65504, 1e-7, 3e9, -3e9, 2.5, -2.5],
                                 np.float32)])
    b = np.concatenate([np.arange(64, -64, -1, dtype=np.float32) * 0.5,
                        rng.standard_normal(n) * 8,
                        np.array([1.0, np.nan, 2.0, -0.0, 0.0, 3, -40, 200, 5, 129, 2.5, 2.0], np.float32)])
    # PE buffers hold values loaded from the fp16 G-buffer (large values overflow to inf there)
    with np.errstate(over="ignore"):
        return a.astype(np.float16).astype(np.float32), b.astype(np.float16).astype(np.float32)


@pytest.mark.parametrize("word", WORDS + EXTRA, ids=[hex(w) for w in WORDS + EXTRA])
def test_isa_instruction(cuda_device, word):
    rng = np.random.default_rng(word & 0xFFFF)
    a, b = inputs(rng)
    prev = (rng.standard_normal(a.size) * 10).astype(np.float32)
    exp = cmodel.vector_op(word, a, b, prev)
    t = lambda x: torch.from_numpy(x).to(cuda_device)  # noqa: E731
    got = nb.isa_vector(word, t(a), t(b), t(prev)).cpu().numpy()
    op = word & 0xFF
    transcendental = op == 0x0F or ((word >> 29) & 1 and 0x40 <= op <= 0x43)
    if not transcendental:
        # every bit, NaN sign and payload included (the SSE NaN rules of the cmodel's host)
        same = got.view(np.uint32) == exp.view(np.uint32)
        assert same.all(), (hex(word), a[~same][:4], b[~same][:4], got[~same][:4], exp[~same][:4])
    else:
        fin = np.isfinite(exp)
        assert np.array_equal(np.isfinite(got), fin)
        ulp = np.abs(got[fin].view(np.int32).astype(np.int64) - exp[fin].view(np.int32).astype(np.int64))
        assert ulp.max() <= 4


def test_fp16_store_rounding_bit_exact(cuda_device):
    rng = np.random.default_rng(5)
    bits = rng.integers(0, 2 ** 32, 1 << 20, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    got = nb.f32_to_f16_bits(torch.from_numpy(x).to(cuda_device)).cpu().numpy().view(np.uint16)
    assert np.array_equal(got, cmodel.f32_to_f16_bits(x))
    back = nb.f16_bits_to_f32(torch.from_numpy(got.view(np.int16)).to(cuda_device)).cpu().numpy()
    # the cmodel's widening keeps a NaN's sign and payload (sign | 0x7F800000 | m << 13)
    assert np.array_equal(back.view(np.uint32), got.view(np.float16).astype(np.float32).view(np.uint32))

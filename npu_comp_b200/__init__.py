"""npu_comp_b200 -- B200 (sm_100a) implementation of the compute that the
KwanyoungCho/NPU_COMP compiler lowers onto its NPU: the W8A16 matmul and the
Llama-layer ops, behind an operator surface named after
b_program_examples/npu.py.  Kernels live in libnpub.so (C ABI: include/npub.h).
"""
from .npu import (  # noqa: F401
    NpubError, add, argmax, attention, attention_decode, embed, f16_bits_to_f32, f32_to_f16_bits, fp16, isa_vector, kv_append, matmul,
    quantize_w8, rmsnorm, rope, rope_freqs, rope_kv_append, rope_kv_store, softmax, swiglu, matmul_swiglu,
    interleave_gate_up, matmul_rms, rmsnorm_parts,
)

from .llama import llama_layer  # noqa: F401,E402
from . import checkpoint, frontend  # noqa: F401,E402

__version__ = "1.0.0"

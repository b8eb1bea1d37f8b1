"""The C ABI library (CPU): it loads, exports every entry point declared in
include/npub.h, and rejects invalid arguments with NPUB_ERR_INVALID_ARG before
touching a device."""
import ctypes
import os
import re

import pytest

from npu_comp_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    src = open(os.path.join(ROOT, "include", "npub.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(npub_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_bound_entry_points():
    names = declared()
    assert len(names) >= 20
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol(libnpub_path):
    lib = ctypes.CDLL(libnpub_path)
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_status_strings_and_version(libnpub_path):
    lib = _lib.load()
    assert lib.npub_version() >= 10000
    for st in (0, -1, -2, -3, -4, -5, -6):
        assert lib.npub_strerror(st)
    assert lib.npub_strerror(-1).decode().startswith("invalid argument")


def test_invalid_arguments_rejected_before_any_device_work(libnpub_path):
    lib = _lib.load()
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    # K not a multiple of 16
    assert lib.npub_w8a16_gemm(p, 24, p, 32, None, p, 8, None, 0, 4, 8, 24, 1.0, None, 0, None) == -1
    # lda < K
    assert lib.npub_w8a16_gemm(p, 8, p, 32, None, p, 8, None, 0, 4, 8, 16, 1.0, None, 0, None) == -1
    # misaligned activation pointer
    assert lib.npub_f16_gemm(ctypes.c_void_p(18), 16, p, 16, None, p, 8, None, 0, 4, 8, 16, 1.0, None, 0,
                             None) == -1
    # d not a multiple of 8
    assert lib.npub_rmsnorm(p, 12, None, 0, None, 0, p, p, 12, 2, 12, 1e-5, None) == -1
    # heads not divisible by kv_heads
    assert lib.npub_attention_prefill(p, 384, p, 256, p, 256, p, 384, 1, 8, 3, 2, 128, 0.1, 1, p, 1 << 30,
                                      None) == -1
    # unsupported head_dim for decode
    assert lib.npub_attention_decode(p, 64, p, p, 16, None, 8, p, 64, 1, 1, 1, 64, 0.1, None, 0, None) == -2
    # matrix multiply is not an elementwise instruction
    assert lib.npub_isa_vector((2 << 30) | 0x42, p, p, None, p, 4, None) == -2
    # zero-sized work is a no-op
    assert lib.npub_swiglu(None, 0, None, 0, None, 0, 0, 0, None) == 0


def test_python_wrappers_fail_loudly_without_the_library(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(ImportError):
        _lib.load(str(tmp_path / "missing.so"))


def test_fused_entry_points_validate_before_any_device_work(libnpub_path):
    """The gate|up + SwiGLU GEMM and the prompt RoPE + KV-store reject bad
    shapes with NPUB_ERR_INVALID_ARG and treat empty work as a no-op."""
    lib = _lib.load()
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    # npub_w8a16_gemm_swiglu(A, lda, Wq, ldw, scale, C, ldc, M, F, K, ws, ws_bytes, stream)
    assert lib.npub_w8a16_gemm_swiglu(p, 24, p, 32, None, p, 8, 4, 8, 24, None, 0, None) == -1  # K % 16
    assert lib.npub_w8a16_gemm_swiglu(p, 16, p, 16, None, p, 4, 4, 8, 16, None, 0, None) == -1  # ldc < F
    assert lib.npub_w8a16_gemm_swiglu(p, 16, ctypes.c_void_p(24), 16, None, p, 8, 4, 8, 16, None, 0,
                                      None) == -1  # misaligned weights
    assert lib.npub_w8a16_gemm_swiglu(None, 0, None, 0, None, None, 0, 0, 8, 16, None, 0, None) == 0  # M == 0
    # npub_rope_kv_store(qkv, ldx, tokens, tokens_per_seq, hq, hk, hd, positions, theta, kc, vc, cap, stream)
    assert lib.npub_rope_kv_store(p, 512, 10, 3, 2, 1, 128, p, 1e4, p, p, 16, None) == -1  # ragged sequences
    assert lib.npub_rope_kv_store(p, 512, 8, 4, 2, 1, 120, p, 1e4, p, p, 16, None) == -1  # head_dim % 16
    assert lib.npub_rope_kv_store(p, 256, 8, 4, 2, 1, 128, p, 1e4, p, p, 16, None) == -1  # ldx too small
    assert lib.npub_rope_kv_store(None, 0, 0, 1, 2, 1, 128, None, 1e4, None, None, 0, None) == 0  # no rows


def test_folded_norm_entry_points_validate_before_any_device_work(libnpub_path):
    """The RMSNorm-folded decode GEMM, its input kernel and the norm-folding
    all-reduce reject bad shapes before touching a device; empty work is a
    no-op and more than 64 tokens is NPUB_ERR_UNSUPPORTED."""
    lib = _lib.load()
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    f = ctypes.c_float(1e-5)

    def rms(A, lda, M, N, K, swiglu=0, rs=None, rs_n=0, rs_ld=0, rs_d=0, gamma=None, G=None, ldg=0, ss=None,
            ss_ld=0, R=None, ldr=0, ldc=None):
        return lib.npub_w8a16_gemm_rms(A, lda, p, 16 * ((K + 15) // 16), p, p, ldc if ldc is not None else N, R,
                                       ldr, M, N, K, swiglu, rs, rs_n, rs_ld, rs_d, f, gamma, G, ldg, ss, ss_ld,
                                       None, 0, 0, 0, None, 0, None)
    assert rms(p, 16, 0, 128, 16) == 0                          # no tokens
    assert rms(p, 16, 65, 128, 16) == -2                        # more than 64 tokens
    assert rms(p, 24, 4, 128, 24) == -1                         # K % 16
    assert rms(p, 16, 4, 128, 16, rs=p, rs_n=4, rs_ld=2, rs_d=128) == -1   # rs_ld < M
    assert rms(p, 16, 4, 128, 16, G=p, gamma=None, ldg=128) == -1          # G without gamma
    assert rms(p, 16, 4, 100, 16, ss=p, ss_ld=4) == -1                     # N % 32 with ss
    assert rms(p, 16, 4, 128, 16, swiglu=1, R=p, ldr=128) == -1            # SwiGLU with a residual
    # npub_rmsnorm_parts(x, ldx, gamma, G, ldg, ss, ss_ld, rows, d, stream)
    assert lib.npub_rmsnorm_parts(p, 48, p, p, 48, p, 4, 4, 48, None) == -1   # d % 32
    assert lib.npub_rmsnorm_parts(p, 64, p, p, 64, p, 2, 4, 64, None) == -1   # ss_ld < rows
    assert lib.npub_rmsnorm_parts(None, 64, None, None, 64, None, 4, 0, 64, None) == 0
    # npub_allreduce_f16_rms(comm, in, out, rows, d, residual, gamma, G, ss, ss_ld, stream)
    assert lib.npub_allreduce_f16_rms(p, p, p, 4, 48, p, p, p, p, 4, None) == -1   # d % 32
    assert lib.npub_allreduce_f16_rms(p, p, p, 4, 64, None, p, p, p, 4, None) == -1  # no residual
    assert lib.npub_allreduce_f16_rms(None, None, None, 0, 64, None, None, None, None, 0, None) == 0

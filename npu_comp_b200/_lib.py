"""ctypes binding of libnpub.so (the C ABI declared in include/npub.h).

The library is loaded from the package directory; when it is missing the
import of any operator fails loudly -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libnpub.so")

NPUB_OK = 0
NPUB_ERR_INVALID_ARG = -1
NPUB_ERR_UNSUPPORTED = -2
NPUB_ERR_CUDA = -3
NPUB_ERR_WORKSPACE = -4
NPUB_ERR_DEVICE_TIMEOUT = -5
NPUB_ERR_NO_DEVICE = -6
NPUB_ERR_SCRATCH_LIMIT = -7
NPUB_NO_CAUSAL = -1

_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float
_sz = ctypes.c_size_t
_u32 = ctypes.c_uint32

# name -> (restype, argtypes); must cover every function declared in include/npub.h
SIGNATURES = {
    "npub_version": (_i, []),
    "npub_strerror": (ctypes.c_char_p, [_i]),
    "npub_last_cuda_error": (_i, []),
    "npub_device_error": (_i, [_i]),
    "npub_launch_count": (ctypes.c_ulonglong, []),
    "npub_w8a16_gemm": (_i, [_p, _i64, _p, _i64, _p, _p, _i64, _p, _i64, _i, _i, _i, _f, _p, _sz, _p]),
    "npub_w8a16_gemm_workspace": (_sz, [_i, _i, _i]),
    "npub_w8a16_gemm_swiglu": (_i, [_p, _i64, _p, _i64, _p, _p, _i64, _i, _i, _i, _p, _sz, _p]),
    "npub_w8a16_gemm_rms": (_i, [_p, _i64, _p, _i64, _p, _p, _i64, _p, _i64, _i, _i, _i, _i,
                                 _p, _i, _i64, _i, _f, _p, _p, _i64, _p, _i64, _p, _i64, _i, _i, _p, _sz, _p]),
    "npub_w8a16_gemm_rms_workspace": (_sz, [_i, _i, _i]),
    "npub_w8a16_kernel_name": (ctypes.c_char_p, [_i, _i, _i]),
    "npub_w8a16_gemm_noalloc": (_i, [_p, _i64, _p, _i64, _p, _p, _i64, _p, _i64, _i, _i, _i, _f, _p]),
    "npub_f16_gemm": (_i, [_p, _i64, _p, _i64, _p, _p, _i64, _p, _i64, _i, _i, _i, _f, _p, _sz, _p]),
    "npub_f16_gemm_workspace": (_sz, [_i, _i, _i]),
    "npub_quantize_w8": (_i, [_p, _i64, _i, _i, _p, _i64, _p, _p]),
    "npub_rmsnorm": (_i, [_p, _i64, _p, _i64, _p, _i64, _p, _p, _i64, _i, _i, _f, _p]),
    "npub_rmsnorm_parts": (_i, [_p, _i64, _p, _p, _i64, _p, _i64, _i, _i, _p]),
    "npub_swiglu": (_i, [_p, _i64, _p, _i64, _p, _i64, _i, _i, _p]),
    "npub_add": (_i, [_p, _i64, _p, _i64, _p, _i64, _i, _i, _p]),
    "npub_embed": (_i, [_p, _i, _p, _i64, _i, _i, _p, _i64, _p]),
    "npub_argmax_rows": (_i, [_p, _i64, _i, _i, _p, _p, _p]),
    "npub_argmax_keys": (_i, [_p, _i64, _i, _i, _i, _p, _p]),
    "npub_select_keys": (_i, [_p, _i, _i, _p, _p]),
    "npub_softmax_rows": (_i, [_p, _p, _i64, _i64, _i, _i, _i, _f, _i, _i, _p]),
    "npub_rope": (_i, [_p, _i64, _i, _i, _i, _p, _i, _f, _p]),
    "npub_attention_prefill": (_i, [_p, _i64, _p, _i64, _p, _i64, _p, _i64, _i, _i, _i, _i, _i, _f, _i, _p, _sz, _p]),
    "npub_attention_workspace": (_sz, [_i, _i, _i, _i]),
    "npub_attention_decode": (_i, [_p, _i64, _p, _p, _i64, _p, _i, _p, _i64, _i, _i, _i, _i, _f, _p, _sz, _p]),
    "npub_attention_decode_workspace": (_sz, [_i, _i, _i, _i]),
    "npub_kv_append": (_i, [_p, _i64, _p, _i64, _p, _p, _i64, _p, _i, _i, _i, _i, _p]),
    "npub_rope_kv_append": (_i, [_p, _i64, _i, _i, _i, _i, _p, _f, _p, _p, _i64, _p, _p]),
    "npub_rope_kv_store": (_i, [_p, _i64, _i, _i, _i, _i, _i, _p, _f, _p, _p, _i64, _p]),
    "npub_rope_freqs": (_i, [_p, _i64, _i, _i, _i, _p, _i, _p, _p]),
    "npub_rope_kv_append_freqs": (_i, [_p, _i64, _i, _i, _i, _i, _p, _p, _p, _p, _i64, _p, _p]),
    "npub_rope_kv_store_freqs": (_i, [_p, _i64, _i, _i, _i, _i, _i, _p, _p, _p, _p, _i64, _p]),
    "npub_rope_llama3_freqs": (_i, [_p, _i, ctypes.c_double, ctypes.c_double, ctypes.c_double, ctypes.c_double,
                                    ctypes.c_double]),
    "npub_isa_vector": (_i, [_u32, _p, _p, _p, _p, _i64, _p]),
    "npub_f32_to_f16": (_i, [_p, _p, _i64, _p]),
    "npub_f16_to_f32": (_i, [_p, _p, _i64, _p]),
    "npub_program_create": (_i, [_p, _i64, _i64, _i64, ctypes.POINTER(ctypes.c_void_p)]),
    "npub_program_error_pc": (_i, []),
    "npub_program_info": (_i, [_p, ctypes.POINTER(ctypes.c_int64), _i]),
    "npub_program_workspace": (_sz, [_p]),
    "npub_program_load": (_i, [_p, _p, _sz, _p]),
    "npub_program_run": (_i, [_p, _p, _i64, _p, _i64, _p, _sz, _p]),
    "npub_program_destroy": (_i, [_p]),
    "npub_comm_handle_bytes": (_sz, []),
    "npub_comm_create": (_i, [_i, _i, _sz, ctypes.POINTER(ctypes.c_void_p), _p]),
    "npub_comm_open": (_i, [_p, _p]),
    "npub_allreduce_f16": (_i, [_p, _p, _p, _i64, _p]),
    "npub_allreduce_f16_rms": (_i, [_p, _p, _p, _i, _i, _p, _p, _p, _p, _i64, _p]),
    "npub_comm_destroy": (_i, [_p]),
}

_lock = threading.Lock()
_lib = None


class NpubError(RuntimeError):
    """A libnpub call returned a non-zero status."""

    def __init__(self, name: str, status: int, text: str):
        super().__init__(f"{name} failed: {text} (status {status})")
        self.status = status


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load libnpub.so once and bind every entry point's signature."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise ImportError(
                f"libnpub.so not found at {path}: build it with `python -m npu_comp_b200.build` "
                "(there is no CPU fallback)")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def call(name: str, *args) -> None:
    """Call an npub_* function and raise on a non-zero status."""
    lib = load()
    st = getattr(lib, name)(*args)
    if st != NPUB_OK:
        text = lib.npub_strerror(st).decode()
        if st == NPUB_ERR_CUDA:
            text += f" (cudaError {lib.npub_last_cuda_error()})"
        if st == NPUB_ERR_INVALID_ARG:
            raise ValueError(f"{name}: {text}")
        raise NpubError(name, st, text)


def launch_count() -> int:
    """Kernels launched by libnpub so far in this process."""
    return int(load().npub_launch_count())


def query(name: str, *args) -> int:
    return int(getattr(load(), name)(*args))

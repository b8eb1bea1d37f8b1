"""Operator surface of the B200 build, named after the reference's
`b_program_examples/npu.py` (fp16, matmul, run) and the Llama-layer macros of
`b_program_examples/llama_layer.py:71-152` (rmsnorm, rope, attention, FFN).

Where the reference's functions *emit NPU instructions* that mysim later
executes (npu.py:41-47 appends an m_mul program; npu.py:62-71 runs it), these
functions *compute*: they take CUDA tensors, launch the sm_100a kernels of
libnpub.so on the current stream and return CUDA tensors.  Every op calls the
C ABI of include/npub.h through ctypes; there is no CPU or PyTorch fallback.

Errors: invalid shapes/dtypes raise ValueError (the reference raises
CodegenError, d_compiler/npu_compiler/codegen.py:21-22); a failing CUDA call
raises NpubError (the reference's CalledProcessError from run()).
"""
from __future__ import annotations

import math
import struct
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import NpubError  # noqa: F401  (re-exported)

__all__ = [
    "fp16", "quantize_w8", "matmul", "rmsnorm", "add", "swiglu", "softmax", "rope", "attention",
    "attention_decode", "kv_append", "rope_kv_append", "rope_kv_store", "matmul_swiglu", "interleave_gate_up",
    "matmul_rms", "rmsnorm_parts",
    "embed", "argmax", "isa_vector", "f32_to_f16_bits", "f16_bits_to_f32", "device_error", "NpubError",
]


def fp16(x: float) -> float:
    """Round a python float through FP16 (b_program_examples/npu.py:7-8)."""
    return struct.unpack('<e', struct.pack('<e', float(x)))[0]


# ----------------------------------------------------------------- helpers

def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _mat(t: torch.Tensor, name: str, dtype: torch.dtype) -> int:
    """Validate a row-major CUDA matrix and return its leading dimension."""
    _need(isinstance(t, torch.Tensor), f"{name} must be a torch.Tensor")
    _need(t.is_cuda, f"{name} must be a CUDA tensor")
    _need(t.dtype == dtype, f"{name} must be {dtype}, got {t.dtype}")
    _need(t.dim() == 2, f"{name} must be 2-D, got shape {tuple(t.shape)}")
    _need(t.stride(1) == 1 or t.shape[1] == 1, f"{name} must have unit stride along its last dim")
    return max(t.stride(0), t.shape[1]) if t.shape[0] <= 1 else t.stride(0)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _workspace(nbytes: int, device) -> Tuple[Optional[torch.Tensor], int]:
    if nbytes <= 0:
        return None, 0
    ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=device)
    off = (-ws.data_ptr()) % 256
    return ws[off:off + nbytes], nbytes


# A W8A16 workspace starts with 64 KiB of tile counters for the few-token
# (stream-K) kernel; they must start at zero and every call leaves them at
# zero.  One zero-filled buffer per (device, stream) serves every W8A16 call;
# a grown buffer replaces the old one, which is kept alive for CUDA graphs
# that captured its address.
_zeroed_ws = {}
_retired_ws = []


def device_error(clear: bool = False) -> int:
    """The current device's error word: non-zero when a bounded device-side wait
    gave up (NPUB_ERR_DEVICE_TIMEOUT cases; synchronises the device).

    With clear=True the word is reset, and so are the tile counters of every
    W8A16 workspace this module hands out and of the library's allocation-free
    scratch: a stream-K call whose wait gave up may have left counts there,
    which the next call would take for pieces already written."""
    lib = _lib.load()
    v = int(lib.npub_device_error(1 if clear else 0))
    if v == _lib.NPUB_ERR_CUDA:
        raise NpubError("npub_device_error", v, lib.npub_strerror(v).decode())
    if clear:
        dev = torch.cuda.current_device()
        for (d, _), buf in _zeroed_ws.items():
            if d == dev:
                buf.zero_()
        torch.cuda.synchronize()
    return v


def _zeroed_workspace(nbytes: int, device) -> Tuple[Optional[torch.Tensor], int]:
    if nbytes <= 0:
        return None, 0
    key = (device.index if device.index is not None else torch.cuda.current_device(), _stream())
    buf = _zeroed_ws.get(key)
    if buf is None or buf.numel() < nbytes:
        if buf is not None:
            _retired_ws.append(buf)
        buf = torch.zeros(max(nbytes, 4 << 20), dtype=torch.uint8, device=device)
        _zeroed_ws[key] = buf
    return buf, buf.numel()


# -------------------------------------------------------------- W8A16 matmul

# When a list, every matmul() call appends (start_event, end_event, flops, int8)
# recorded on the launching stream -- used by bench.py to time the GEMM kernels
# inside a step.
gemm_events = None



def quantize_w8(W: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Symmetric per-output-channel int8 quantisation of W [K, N] fp32 (x @ W).

    Returns (Wq int8 [N, K] K-major, scale fp16 [N]) with
    scale[n] = fp16(max_k |W[k, n]| / 127) and Wq[n, k] = clip(rint(W[k, n] / scale[n]), +-127).
    """
    ldw = _mat(W, "W", torch.float32)
    K, N = W.shape
    q = torch.empty((N, K), dtype=torch.int8, device=W.device)
    s = torch.empty((N,), dtype=torch.float16, device=W.device)
    _lib.call("npub_quantize_w8", W.data_ptr(), ldw, K, N, q.data_ptr(), K, s.data_ptr(), _stream())
    return q, s


def matmul(A: torch.Tensor, W: torch.Tensor, scale: Optional[torch.Tensor] = None, *,
           out: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None,
           alpha: float = 1.0) -> torch.Tensor:
    """C[M, N] = fp16(alpha * scale[n] * sum_k A[m, k] W[n, k]) (+ residual[m, n]).

    The reference's matmul (npu.py:41-47) computes C = A @ B with B [K, N]; here
    the weight is packed K-major as W [N, K] -- int8 (W8A16, from quantize_w8)
    or fp16 (W = B.T.contiguous()).  A is fp16 [M, K]; K must be a multiple of 16.
    """
    lda = _mat(A, "A", torch.float16)
    _need(W.dtype in (torch.int8, torch.float16), "W must be int8 or float16")
    ldw = _mat(W, "W", W.dtype)
    M, K = A.shape
    N, K2 = W.shape
    _need(K == K2, f"K mismatch: A {tuple(A.shape)} vs W {tuple(W.shape)}")
    if scale is not None:
        _need(scale.is_cuda and scale.dtype == torch.float16 and scale.numel() == N and scale.is_contiguous(),
              "scale must be a contiguous fp16 CUDA tensor of N elements")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=A.device)
    ldc = _mat(out, "out", torch.float16)
    _need(tuple(out.shape) == (M, N), "out must be [M, N]")
    ldr = 0
    if residual is not None:
        ldr = _mat(residual, "residual", torch.float16)
        _need(tuple(residual.shape) == (M, N), "residual must be [M, N]")
    int8 = W.dtype == torch.int8
    wsq = "npub_w8a16_gemm_workspace" if int8 else "npub_f16_gemm_workspace"
    if int8:
        ws, wsb = _zeroed_workspace(_lib.query(wsq, M, N, K), A.device)
    else:
        ws, wsb = _workspace(_lib.query(wsq, M, N, K), A.device)
    fn = "npub_w8a16_gemm" if int8 else "npub_f16_gemm"
    ev = gemm_events
    if ev is not None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
    _lib.call(fn, A.data_ptr(), lda, W.data_ptr(), ldw, _ptr(scale), out.data_ptr(), ldc, _ptr(residual), ldr,
              M, N, K, float(alpha), _ptr(ws), wsb, _stream())
    if ev is not None:
        e1.record()
        ev.append((e0, e1, 2.0 * M * N * K, int8))
    return out


def interleave_gate_up(wq: torch.Tensor, scale: torch.Tensor):
    """[gate rows (F) | up rows (F)] -> rows 2c = gate c, 2c + 1 = up c, the
    layout matmul_swiglu takes (int8 [2F, K] and fp16 [2F])."""
    F2, K = wq.shape
    _need(F2 % 2 == 0 and scale.numel() == F2, "gate|up weights need an even row count and one scale per row")
    F = F2 // 2
    w = wq.view(2, F, K).transpose(0, 1).reshape(F2, K).contiguous()
    s = scale.view(2, F).t().reshape(F2).contiguous()
    return w, s


def matmul_swiglu(A: torch.Tensor, Wgu: torch.Tensor, scale: torch.Tensor, *,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[M, F] = fp16(silu(g) * u) with g, u the fp16 W8A16 projections of A
    on the gate and up rows of Wgu (int8 [2F, K], interleaved by
    interleave_gate_up; scale fp16 [2F]): matmul() then swiglu(), fused."""
    lda = _mat(A, "A", torch.float16)
    ldw = _mat(Wgu, "Wgu", torch.int8)
    M, K = A.shape
    F2, K2 = Wgu.shape
    _need(K == K2 and F2 % 2 == 0, f"shape mismatch: A {tuple(A.shape)} vs Wgu {tuple(Wgu.shape)}")
    _need(scale.is_cuda and scale.dtype == torch.float16 and scale.numel() == F2 and scale.is_contiguous(),
          "scale must be a contiguous fp16 CUDA tensor of 2F elements")
    F = F2 // 2
    if out is None:
        out = torch.empty((M, F), dtype=torch.float16, device=A.device)
    ldo = _mat(out, "out", torch.float16)
    _need(tuple(out.shape) == (M, F), "out must be [M, F]")
    ws, wsb = _zeroed_workspace(_lib.query("npub_w8a16_gemm_workspace", M, F2, K), A.device)
    ev = gemm_events
    if ev is not None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
    _lib.call("npub_w8a16_gemm_swiglu", A.data_ptr(), lda, Wgu.data_ptr(), ldw, scale.data_ptr(), out.data_ptr(),
              ldo, M, F, K, _ptr(ws), wsb, _stream())
    if ev is not None:
        e1.record()
        ev.append((e0, e1, 2.0 * M * F2 * K, True))
    return out


def matmul_rms(A: torch.Tensor, Wq: torch.Tensor, scale: torch.Tensor, *, out: Optional[torch.Tensor] = None,
               residual: Optional[torch.Tensor] = None, swiglu: bool = False,
               rs: Optional[Tuple[torch.Tensor, int]] = None, eps: float = 1e-5,
               gamma: Optional[torch.Tensor] = None, g_out: Optional[torch.Tensor] = None,
               ss_out: Optional[torch.Tensor] = None, prefetch_next: Optional[torch.Tensor] = None):
    """W8A16 GEMM of a decode step (M <= 64) with an RMSNorm folded in
    (npub_w8a16_gemm_rms): the RMSNorm -> projection pairs of a decode layer
    without the normalised activations' round trip or their own launch.

    rs=(ss, d): A is fp16(h * gamma) of a residual stream h (rmsnorm_parts or a
    producer call below) and row t of the result is scaled by
    1 / sqrt(sum(ss[:, t]) / d + eps) before rounding (before SwiGLU with
    swiglu=True, where Wq holds interleaved gate/up rows and out is [M, N/2]).
    gamma: also return (out, g_out, ss_out) -- g_out = fp16(out * gamma) and
    ss_out [N/32, M] fp32, the next call's rs.  prefetch_next: the int8 weights
    of the next GEMM of a decode chain (same M), whose first tiles go to L2
    while this GEMM runs.  Raises NpubError for M > 64."""
    lda = _mat(A, "A", torch.float16)
    ldw = _mat(Wq, "Wq", torch.int8)
    M, K = A.shape
    N, K2 = Wq.shape
    _need(K == K2, f"K mismatch: A {tuple(A.shape)} vs Wq {tuple(Wq.shape)}")
    _need(scale.is_cuda and scale.dtype == torch.float16 and scale.numel() == N and scale.is_contiguous(),
          "scale must be a contiguous fp16 CUDA tensor of N elements")
    NC = N // 2 if swiglu else N
    if out is None:
        out = torch.empty((M, NC), dtype=torch.float16, device=A.device)
    ldc = _mat(out, "out", torch.float16)
    _need(tuple(out.shape) == (M, NC), f"out must be [{M}, {NC}]")
    ldr = 0
    if residual is not None:
        ldr = _mat(residual, "residual", torch.float16)
        _need(tuple(residual.shape) == (M, N), "residual must be [M, N]")
    rs_p, rs_n, rs_ld, rs_d = None, 0, 0, 0
    if rs is not None:
        ss, rs_d = rs
        _need(ss.is_cuda and ss.dtype == torch.float32 and ss.dim() == 2 and ss.shape[1] >= M and ss.stride(1) == 1,
              "rs[0] must be fp32 CUDA [parts, >= M] with unit column stride")
        rs_p, rs_n, rs_ld = ss, ss.shape[0], ss.stride(0)
    ldg = ss_ld = 0
    if gamma is not None:
        _need(gamma.is_cuda and gamma.dtype == torch.float16 and gamma.numel() == N and gamma.is_contiguous(),
              "gamma must be a contiguous fp16 CUDA tensor of N elements")
        if g_out is None:
            g_out = torch.empty((M, N), dtype=torch.float16, device=A.device)
        if ss_out is None:
            ss_out = torch.empty((N // 32, M), dtype=torch.float32, device=A.device)
        ldg = _mat(g_out, "g_out", torch.float16)
        _need(ss_out.dtype == torch.float32 and ss_out.dim() == 2 and ss_out.shape[0] == N // 32 and
              ss_out.shape[1] >= M and ss_out.stride(1) == 1, "ss_out must be fp32 [N/32, >= M]")
        ss_ld = ss_out.stride(0)
    ws, wsb = _zeroed_workspace(_lib.query("npub_w8a16_gemm_rms_workspace", M, N, K), A.device)
    _lib.call("npub_w8a16_gemm_rms", A.data_ptr(), lda, Wq.data_ptr(), ldw, scale.data_ptr(), out.data_ptr(), ldc,
              _ptr(residual), ldr, M, N, K, 1 if swiglu else 0, _ptr(rs_p), rs_n, rs_ld, int(rs_d), float(eps),
              _ptr(gamma), _ptr(g_out if gamma is not None else None), ldg,
              _ptr(ss_out if gamma is not None else None), ss_ld, _ptr(prefetch_next),
              prefetch_next.stride(0) if prefetch_next is not None else 0,
              prefetch_next.shape[0] if prefetch_next is not None else 0,
              prefetch_next.shape[1] if prefetch_next is not None else 0, _ptr(ws), wsb, _stream())
    return out if gamma is None else (out, g_out, ss_out)


def rmsnorm_parts(x: torch.Tensor, gamma: torch.Tensor, *, g_out: Optional[torch.Tensor] = None,
                  ss_out: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """The (g, ss) that matmul_rms(rs=(ss, d)) takes for an RMSNorm of x
    (fp16 [rows, d], d % 32 == 0): g = fp16(x * gamma), ss [d/32, rows] fp32
    the sums of x^2 over every 32 columns."""
    ldx = _mat(x, "x", torch.float16)
    rows, d = x.shape
    _need(gamma.is_cuda and gamma.dtype == torch.float16 and gamma.numel() == d and gamma.is_contiguous(),
          "gamma must be a contiguous fp16 CUDA tensor of d elements")
    if g_out is None:
        g_out = torch.empty((rows, d), dtype=torch.float16, device=x.device)
    if ss_out is None:
        ss_out = torch.empty((d // 32, rows), dtype=torch.float32, device=x.device)
    ldg = _mat(g_out, "g_out", torch.float16)
    _need(ss_out.dtype == torch.float32 and ss_out.dim() == 2 and ss_out.shape[0] == d // 32 and
          ss_out.shape[1] >= rows and ss_out.stride(1) == 1, "ss_out must be fp32 [d/32, >= rows]")
    _lib.call("npub_rmsnorm_parts", x.data_ptr(), ldx, gamma.data_ptr(), g_out.data_ptr(), ldg, ss_out.data_ptr(),
              ss_out.stride(0), rows, d, _stream())
    return g_out, ss_out


# ---------------------------------------------------------------- vector ops

def rmsnorm(x: torch.Tensor, gamma: torch.Tensor, eps: float = 1e-5, *, residual: Optional[torch.Tensor] = None,
            residual_out: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None):
    """y = fp16(x / sqrt(mean(x^2) + eps) * gamma) per row (legalize.py:30-47).

    With `residual`, h = fp16(x + residual) is formed first (llama_layer.py:139),
    written to `residual_out` (default: a new tensor) and normalised; returns (y, h).
    """
    ldx = _mat(x, "x", torch.float16)
    rows, d = x.shape
    _need(gamma.is_cuda and gamma.dtype == torch.float16 and gamma.numel() == d and gamma.is_contiguous(),
          "gamma must be a contiguous fp16 CUDA tensor of d elements")
    if out is None:
        out = torch.empty((rows, d), dtype=torch.float16, device=x.device)
    ldy = _mat(out, "out", torch.float16)
    ldr = ldxo = 0
    if residual is not None:
        ldr = _mat(residual, "residual", torch.float16)
        _need(tuple(residual.shape) == (rows, d), "residual must match x")
        if residual_out is None:
            residual_out = torch.empty((rows, d), dtype=torch.float16, device=x.device)
        ldxo = _mat(residual_out, "residual_out", torch.float16)
    _lib.call("npub_rmsnorm", x.data_ptr(), ldx, _ptr(residual), ldr, _ptr(residual_out), ldxo, gamma.data_ptr(),
              out.data_ptr(), ldy, rows, d, float(eps), _stream())
    return out if residual is None else (out, residual_out)


def add(a: torch.Tensor, b: torch.Tensor, *, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out = fp16(a + b), the residual add of llama_layer.py:139,152 (fp16 [rows, cols])."""
    lda = _mat(a, "a", torch.float16)
    ldb = _mat(b, "b", torch.float16)
    _need(a.shape == b.shape, "a and b must have the same shape")
    rows, cols = a.shape
    if out is None:
        out = torch.empty((rows, cols), dtype=torch.float16, device=a.device)
    ldo = _mat(out, "out", torch.float16)
    _lib.call("npub_add", a.data_ptr(), lda, b.data_ptr(), ldb, out.data_ptr(), ldo, rows, cols, _stream())
    return out


def swiglu(g: torch.Tensor, u: Optional[torch.Tensor] = None, *, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """h = fp16(g / (1 + exp(-g)) * u) (legalize.py:130-149).  With u=None, g is
    [rows, 2F] holding the gate in its first F columns and up in the last F."""
    if u is None:
        _need(g.dim() == 2 and g.shape[1] % 2 == 0, "g must be [rows, 2F] when u is None")
        F = g.shape[1] // 2
        g, u = g[:, :F], g[:, F:]
    ldg = _mat(g, "g", torch.float16)
    ldu = _mat(u, "u", torch.float16)
    _need(g.shape == u.shape, "g and u must have the same shape")
    rows, cols = g.shape
    if out is None:
        out = torch.empty((rows, cols), dtype=torch.float16, device=g.device)
    ldh = _mat(out, "out", torch.float16)
    _lib.call("npub_swiglu", g.data_ptr(), ldg, u.data_ptr(), ldu, out.data_ptr(), ldh, rows, cols, _stream())
    return out


def softmax(s: torch.Tensor, *, causal: bool = False, scale: float = 1.0, causal_offset: int = 0,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Row softmax of scale*s over the last dim (legalize.py:97-114); causal rows
    r see columns c <= r + causal_offset and get exact zeros elsewhere."""
    _need(s.is_cuda and s.dtype == torch.float16 and s.dim() >= 2 and s.is_contiguous(),
          "s must be a contiguous fp16 CUDA tensor with >= 2 dims")
    rows, cols = s.shape[-2], s.shape[-1]
    batch = s.numel() // max(1, rows * cols)
    _need(cols % 8 == 0, "the row length must be a multiple of 8")
    if out is None:
        out = torch.empty_like(s)
    _need(out.shape == s.shape and out.is_contiguous() and out.dtype == torch.float16, "bad out")
    _lib.call("npub_softmax_rows", s.data_ptr(), out.data_ptr(), cols, rows * cols, batch, rows, cols, float(scale),
              int(causal_offset) if causal else _lib.NPUB_NO_CAUSAL, 1, _stream())
    return out


def _freq_table(inv_freq: Optional[torch.Tensor], head_dim: int, dev) -> Optional[int]:
    if inv_freq is None:
        return None
    _need(inv_freq.is_cuda and inv_freq.device == dev and inv_freq.dtype == torch.float32
          and inv_freq.is_contiguous() and inv_freq.numel() == head_dim // 2,
          "inv_freq must be contiguous fp32 CUDA [head_dim/2] on the tensor's device")
    return inv_freq.data_ptr()


def rope_freqs(head_dim: int, theta: float = 10000.0, *, llama3_scaling=None, device=None) -> torch.Tensor:
    """Per-frequency rates [head_dim/2] (fp32) for the *_freqs RoPE paths:
    theta^(-2i/head_dim), with the Llama-3 frequency scaling of
    legalize.py:50-64 when llama3_scaling is True (the reference's factor 32,
    low 1, high 4, old context 8192) or a tuple (factor, low, high, old_ctx).
    Built on the host by npub_rope_llama3_freqs, then copied to `device`."""
    import ctypes
    if llama3_scaling is True:
        llama3_scaling = (32.0, 1.0, 4.0, 8192.0)
    factor, low, high, old = llama3_scaling if llama3_scaling else (0.0, 1.0, 4.0, 8192.0)
    out = (ctypes.c_float * (head_dim // 2))()
    _lib.call("npub_rope_llama3_freqs", ctypes.addressof(out), int(head_dim), float(theta), float(factor), float(low),
              float(high), float(old))
    t = torch.tensor(list(out), dtype=torch.float32)
    return t.to(device) if device is not None else t


def rope(x: torch.Tensor, heads: int, head_dim: int, *, pos0: int = 0, positions: Optional[torch.Tensor] = None,
         theta: float = 10000.0, inv_freq: Optional[torch.Tensor] = None) -> torch.Tensor:
    """In-place RoPE on the first heads*head_dim columns of x [tokens, >=heads*head_dim]
    (rotate_half convention, llama_layer.py:33-40,96-112).  inv_freq (fp32
    CUDA [head_dim/2], from rope_freqs) replaces theta's frequencies, e.g.
    the Llama-3 scaled ones.  Returns x."""
    ldx = _mat(x, "x", torch.float16)
    tokens = x.shape[0]
    _need(x.shape[1] >= heads * head_dim, "x is narrower than heads*head_dim")
    pos_ptr = None
    if positions is not None:
        _need(positions.is_cuda and positions.dtype == torch.int32 and positions.numel() == tokens
              and positions.is_contiguous(), "positions must be contiguous int32 CUDA [tokens]")
        pos_ptr = positions.data_ptr()
    fp = _freq_table(inv_freq, head_dim, x.device)
    if fp is None:
        _lib.call("npub_rope", x.data_ptr(), ldx, tokens, heads, head_dim, pos_ptr, int(pos0), float(theta),
                  _stream())
    else:
        _lib.call("npub_rope_freqs", x.data_ptr(), ldx, tokens, heads, head_dim, pos_ptr, int(pos0), fp, _stream())
    return x


# ------------------------------------------------------- embedding / argmax

def embed(ids: torch.Tensor, table: torch.Tensor, *, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Rows of the fp16 embedding table [vocab, d] for int32 token ids [n]."""
    _need(ids.is_cuda and ids.dtype == torch.int32 and ids.is_contiguous(), "ids must be contiguous int32 CUDA")
    ldt = _mat(table, "table", torch.float16)
    vocab, d = table.shape
    n = ids.numel()
    if out is None:
        out = torch.empty((n, d), dtype=torch.float16, device=table.device)
    ldo = _mat(out, "out", torch.float16)
    _lib.call("npub_embed", ids.data_ptr(), n, table.data_ptr(), ldt, vocab, d, out.data_ptr(), ldo, _stream())
    return out


def argmax(x: torch.Tensor, *, idx: Optional[torch.Tensor] = None, val: Optional[torch.Tensor] = None):
    """Per-row (index, value) of the largest fp16 logit (smallest index on ties)."""
    ldx = _mat(x, "x", torch.float16)
    rows, cols = x.shape
    if idx is None:
        idx = torch.empty((rows,), dtype=torch.int32, device=x.device)
    if val is None:
        val = torch.empty((rows,), dtype=torch.float32, device=x.device)
    _lib.call("npub_argmax_rows", x.data_ptr(), ldx, rows, cols, idx.data_ptr(), val.data_ptr(), _stream())
    return idx, val


def argmax_keys(x: torch.Tensor, index_offset: int = 0, *, keys: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Per-row greedy key (int64 [rows]) of fp16 logits x: the largest value and
    its smallest index + index_offset in one orderable word (npub_argmax_keys);
    select_keys over the keys of every vocabulary shard gives the global argmax."""
    ldx = _mat(x, "x", torch.float16)
    rows, cols = x.shape
    if keys is None:
        keys = torch.empty((rows,), dtype=torch.int64, device=x.device)
    _need(keys.is_cuda and keys.dtype == torch.int64 and keys.numel() == rows and keys.is_contiguous(),
          "keys must be contiguous int64 CUDA [rows]")
    _lib.call("npub_argmax_keys", x.data_ptr(), ldx, rows, cols, int(index_offset), keys.data_ptr(), _stream())
    return keys


def select_keys(keys: torch.Tensor, ranks: int, *, ids: Optional[torch.Tensor] = None) -> torch.Tensor:
    """ids[b] = index of the largest of keys[r * rows + b] over r < ranks (int32)."""
    _need(keys.is_cuda and keys.dtype == torch.int64 and keys.is_contiguous() and keys.numel() % ranks == 0,
          "keys must be contiguous int64 CUDA [ranks * rows]")
    rows = keys.numel() // ranks
    if ids is None:
        ids = torch.empty((rows,), dtype=torch.int32, device=keys.device)
    _need(ids.is_cuda and ids.dtype == torch.int32 and ids.numel() == rows and ids.is_contiguous(),
          "ids must be contiguous int32 CUDA [rows]")
    _lib.call("npub_select_keys", keys.data_ptr(), int(ranks), rows, ids.data_ptr(), _stream())
    return ids


# ----------------------------------------------------------------- attention

def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, kv_heads: Optional[int] = None, *,
              head_dim: Optional[int] = None, batch: int = 1, causal: bool = True, scale: Optional[float] = None,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Causal (GQA) attention of llama_layer.py:114-137 for `batch` sequences of
    equal length stacked along rows: q [batch*T, heads*hd], k/v [batch*T, kv_heads*hd]."""
    kv_heads = kv_heads or heads
    ldq = _mat(q, "q", torch.float16)
    ldk = _mat(k, "k", torch.float16)
    ldv = _mat(v, "v", torch.float16)
    hd = head_dim or q.shape[1] // heads
    rows = q.shape[0]
    _need(rows % batch == 0, "rows must be a multiple of batch")
    T = rows // batch
    if scale is None:
        scale = 1.0 / math.sqrt(hd)
    if out is None:
        out = torch.empty((rows, heads * hd), dtype=torch.float16, device=q.device)
    ldo = _mat(out, "out", torch.float16)
    ws, wsb = _workspace(_lib.query("npub_attention_workspace", batch, T, heads, hd), q.device)
    _lib.call("npub_attention_prefill", q.data_ptr(), ldq, k.data_ptr(), ldk, v.data_ptr(), ldv, out.data_ptr(), ldo,
              batch, T, heads, kv_heads, hd, float(scale), 1 if causal else 0, _ptr(ws), wsb, _stream())
    return out


def attention_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, *, heads: int,
                     kv_heads: Optional[int] = None, lens: Optional[torch.Tensor] = None, ctx_len: int = 0,
                     scale: Optional[float] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One query token per sequence against fp16 caches [batch, kv_heads, cap, 128]."""
    kv_heads = kv_heads or heads
    ldq = _mat(q, "q", torch.float16)
    batch = q.shape[0]
    _need(k_cache.dim() == 4 and k_cache.shape == v_cache.shape and k_cache.is_contiguous() and
          v_cache.is_contiguous() and k_cache.dtype == torch.float16, "caches must be contiguous fp16 [B, KVH, cap, hd]")
    B, KVH, cap, hd = k_cache.shape
    _need(B == batch and KVH == kv_heads, "cache shape does not match q / kv_heads")
    lens_ptr = None
    if lens is not None:
        _need(lens.is_cuda and lens.dtype == torch.int32 and lens.numel() == batch and lens.is_contiguous(),
              "lens must be contiguous int32 CUDA [batch]")
        lens_ptr = lens.data_ptr()
        ctx = int(ctx_len) if ctx_len else cap
    else:
        ctx = int(ctx_len)
    if scale is None:
        scale = 1.0 / math.sqrt(hd)
    if out is None:
        out = torch.empty((batch, heads * hd), dtype=torch.float16, device=q.device)
    ldo = _mat(out, "out", torch.float16)
    ws, wsb = _workspace(_lib.query("npub_attention_decode_workspace", batch, heads, ctx, hd), q.device)
    _lib.call("npub_attention_decode", q.data_ptr(), ldq, k_cache.data_ptr(), v_cache.data_ptr(), cap, lens_ptr, ctx,
              out.data_ptr(), ldo, batch, heads, kv_heads, hd, float(scale), _ptr(ws), wsb, _stream())
    return out


def kv_append(k_new: torch.Tensor, v_new: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, *,
              pos: Optional[torch.Tensor] = None, pos0: int = 0) -> None:
    """cache[b, h, pos[b], :] = new[b, h*hd:(h+1)*hd] for K and V."""
    ldk = _mat(k_new, "k_new", torch.float16)
    ldv = _mat(v_new, "v_new", torch.float16)
    B, KVH, cap, hd = k_cache.shape
    pos_ptr = None
    if pos is not None:
        _need(pos.is_cuda and pos.dtype == torch.int32 and pos.numel() == B and pos.is_contiguous(),
              "pos must be contiguous int32 CUDA [batch]")
        pos_ptr = pos.data_ptr()
    _lib.call("npub_kv_append", k_new.data_ptr(), ldk, v_new.data_ptr(), ldv, k_cache.data_ptr(), v_cache.data_ptr(),
              cap, pos_ptr, int(pos0), B, KVH, hd, _stream())


# --------------------------------------------------------- NPU ISA semantics

def rope_kv_append(qkv: torch.Tensor, q_heads: int, kv_heads: int, head_dim: int, positions: torch.Tensor,
                   k_cache: torch.Tensor, v_cache: torch.Tensor, *, theta: float = 10000.0,
                   lens: Optional[torch.Tensor] = None, inv_freq: Optional[torch.Tensor] = None) -> None:
    """Decode step: rope() on the q and k heads of the fused QKV rows (in place)
    and kv_append() of the rotated k and the v heads at positions[t], in one
    kernel; lens (int32 [tokens], optional) receives positions + 1."""
    ldx = _mat(qkv, "qkv", torch.float16)
    T = qkv.shape[0]
    _need(qkv.shape[1] >= (q_heads + 2 * kv_heads) * head_dim, "qkv has too few columns")
    _need(positions.is_cuda and positions.dtype == torch.int32 and positions.numel() == T
          and positions.is_contiguous(), "positions must be contiguous int32 CUDA [tokens]")
    for c, n in ((k_cache, "k_cache"), (v_cache, "v_cache")):
        _need(c.is_cuda and c.dtype == torch.float16 and c.is_contiguous() and c.dim() == 4
              and tuple(c.shape[:2]) == (T, kv_heads) and c.shape[3] == head_dim,
              f"{n} must be contiguous fp16 CUDA [tokens, kv_heads, cap, head_dim]")
    if lens is not None:
        _need(lens.is_cuda and lens.dtype == torch.int32 and lens.numel() == T and lens.is_contiguous(),
              "lens must be contiguous int32 CUDA [tokens]")
    fp = _freq_table(inv_freq, head_dim, qkv.device)
    if fp is None:
        _lib.call("npub_rope_kv_append", qkv.data_ptr(), ldx, T, q_heads, kv_heads, head_dim, positions.data_ptr(),
                  float(theta), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[2], _ptr(lens), _stream())
    else:
        _lib.call("npub_rope_kv_append_freqs", qkv.data_ptr(), ldx, T, q_heads, kv_heads, head_dim,
                  positions.data_ptr(), fp, k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[2], _ptr(lens),
                  _stream())


def rope_kv_store(qkv: torch.Tensor, q_heads: int, kv_heads: int, head_dim: int, positions: torch.Tensor,
                  k_cache: torch.Tensor, v_cache: torch.Tensor, *, tokens_per_seq: int,
                  theta: float = 10000.0, inv_freq: Optional[torch.Tensor] = None) -> None:
    """Prefill: rope() on the q and k heads of the fused QKV rows of `batch`
    prompts (rows r = b * tokens_per_seq + i, in place) and the rotated k and the
    v heads written to the caches [batch, kv_heads, cap, head_dim] at
    positions[r], in one kernel."""
    ldx = _mat(qkv, "qkv", torch.float16)
    T = qkv.shape[0]
    _need(tokens_per_seq > 0 and T % tokens_per_seq == 0, "rows must be a whole number of sequences")
    _need(qkv.shape[1] >= (q_heads + 2 * kv_heads) * head_dim, "qkv has too few columns")
    _need(positions.is_cuda and positions.dtype == torch.int32 and positions.numel() == T
          and positions.is_contiguous(), "positions must be contiguous int32 CUDA [tokens]")
    batch = T // tokens_per_seq
    for c, nm in ((k_cache, "k_cache"), (v_cache, "v_cache")):
        _need(c.is_cuda and c.dtype == torch.float16 and c.is_contiguous() and c.dim() == 4
              and tuple(c.shape[:2]) == (batch, kv_heads) and c.shape[3] == head_dim,
              f"{nm} must be contiguous fp16 CUDA [batch, kv_heads, cap, head_dim]")
    fp = _freq_table(inv_freq, head_dim, qkv.device)
    if fp is None:
        _lib.call("npub_rope_kv_store", qkv.data_ptr(), ldx, T, tokens_per_seq, q_heads, kv_heads, head_dim,
                  positions.data_ptr(), float(theta), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[2],
                  _stream())
    else:
        _lib.call("npub_rope_kv_store_freqs", qkv.data_ptr(), ldx, T, tokens_per_seq, q_heads, kv_heads, head_dim,
                  positions.data_ptr(), fp, k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[2], _stream())


def isa_vector(word: int, in1: torch.Tensor, in2: Optional[torch.Tensor] = None,
               prev_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Execute one elementwise NPU compute instruction (_poc/mysim.cpp:114-141)
    over fp32 PE buffers; returns the PE output buffer (fp32)."""
    for t, nm in ((in1, "in1"), (in2, "in2"), (prev_out, "prev_out")):
        if t is not None:
            _need(t.is_cuda and t.dtype == torch.float32 and t.is_contiguous(), f"{nm} must be contiguous fp32 CUDA")
    n = in1.numel()
    out = torch.empty(n, dtype=torch.float32, device=in1.device)
    _lib.call("npub_isa_vector", int(word) & 0xFFFFFFFF, in1.data_ptr(), _ptr(in2), _ptr(prev_out), out.data_ptr(), n,
              _stream())
    return out


def f32_to_f16_bits(x: torch.Tensor) -> torch.Tensor:
    """The cmodel's store rounding (mysim.cpp:19-38): fp32 -> fp16 bit patterns (int16)."""
    _need(x.is_cuda and x.dtype == torch.float32 and x.is_contiguous(), "x must be contiguous fp32 CUDA")
    y = torch.empty(x.shape, dtype=torch.int16, device=x.device)
    _lib.call("npub_f32_to_f16", x.data_ptr(), y.data_ptr(), x.numel(), _stream())
    return y


def f16_bits_to_f32(x: torch.Tensor) -> torch.Tensor:
    _need(x.is_cuda and x.dtype in (torch.int16, torch.float16) and x.is_contiguous(), "x must be 16-bit CUDA")
    y = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    _lib.call("npub_f16_to_f32", x.data_ptr(), y.data_ptr(), x.numel(), _stream())
    return y

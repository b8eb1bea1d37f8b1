"""npub_w8a16_gemm_noalloc: the W8A16 matmul for callers that cannot allocate
device memory (a plugin inside a runtime that owns all device memory, a plain
C/ctypes caller without a device allocator, a fixed-budget decode loop).  It
takes its split-K scratch from a static device array instead of a caller
workspace.  Called here through the C ABI and compared with the allocating
entry point, twice in a row (the array keeps the previous call's contents).

This file is collected last, so a run that stops at the first failure has
already run every other test; it also passes alone in a fresh process.
Tolerance: normwise relative error <= 1e-2 (TOL), as for npub_w8a16_gemm.
"""
import ctypes

import pytest
import torch

import npu_comp_b200 as nb
from npu_comp_b200 import _lib

pytestmark = pytest.mark.gpu
TOL = 1e-2
SCRATCH = 16 << 20  # NPUB_NOALLOC_SCRATCH_BYTES in include/npub.h


def noalloc(A, q, s, out, residual=None, alpha=1.0):
    lib = _lib.load()
    M, K = A.shape
    N = q.shape[0]
    return lib.npub_w8a16_gemm_noalloc(A.data_ptr(), A.stride(0), q.data_ptr(), q.stride(0), s.data_ptr(),
                                       out.data_ptr(), out.stride(0),
                                       None if residual is None else residual.data_ptr(),
                                       0 if residual is None else residual.stride(0), M, N, K, float(alpha),
                                       torch.cuda.current_stream().cuda_stream)


def inputs(M, N, K, dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    W = torch.randn((K, N), generator=g, device=dev) * 0.02
    q, s = nb.quantize_w8(W)
    A = torch.randn((M, K), generator=g, device=dev).half()
    return A, q, s


@pytest.mark.parametrize("M,N,K", [(64, 4096, 4096), (64, 12288, 4096), (200, 300, 160)])
def test_noalloc_matches_workspace_entry_point(cuda_device, M, N, K):
    lib = _lib.load()
    need = lib.npub_w8a16_gemm_workspace(M, N, K)
    assert need <= SCRATCH
    A, q, s = inputs(M, N, K, cuda_device, seed=M + N)
    R = torch.randn((M, N), device=cuda_device).half()
    expect = nb.matmul(A, q, s, residual=R, alpha=0.75).float()
    for call in range(2):
        out = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda_device)
        st = noalloc(A, q, s, out, residual=R, alpha=0.75)
        assert st == 0, lib.npub_strerror(st).decode()
        torch.cuda.synchronize()
        got = out.float()
        e = ((got - expect).abs().max() / expect.abs().max()).item()
        assert e <= TOL, (call, e)
        assert torch.equal(got, expect)  # same kernels, same scratch layout: identical bits


def test_noalloc_scratch_is_exercised_and_reused(cuda_device):
    """A split-K shape really uses the static scratch; a second shape between two
    calls of the first leaves different contents behind, and the result stays right."""
    lib = _lib.load()
    assert lib.npub_w8a16_gemm_workspace(64, 4096, 4096) > 0
    A, q, s = inputs(64, 4096, 4096, cuda_device, seed=1)
    A2, q2, s2 = inputs(64, 12288, 4096, cuda_device, seed=2)
    expect = nb.matmul(A, q, s).float()
    out = torch.empty((64, 4096), dtype=torch.float16, device=cuda_device)
    out2 = torch.empty((64, 12288), dtype=torch.float16, device=cuda_device)
    assert noalloc(A, q, s, out) == 0
    assert noalloc(A2, q2, s2, out2) == 0
    assert noalloc(A, q, s, out) == 0
    torch.cuda.synchronize()
    assert torch.equal(out.float(), expect)


def test_noalloc_rejects_requests_beyond_its_scratch(cuda_device):
    lib = _lib.load()
    shape = None
    for M, N, K in ((256, 8192, 16384), (256, 4096, 32768), (256, 8192, 32768), (128, 8192, 65536)):
        if lib.npub_w8a16_gemm_workspace(M, N, K) > SCRATCH:
            shape = (M, N, K)
            break
    if shape is None:
        pytest.skip("no split-K shape exceeds the scratch on this device")
    M, N, K = shape
    A = torch.zeros((M, K), dtype=torch.float16, device=cuda_device)
    q = torch.zeros((N, K), dtype=torch.int8, device=cuda_device)
    s = torch.zeros((N,), dtype=torch.float16, device=cuda_device)
    out = torch.empty((M, N), dtype=torch.float16, device=cuda_device)
    st = noalloc(A, q, s, out)
    assert st == _lib.NPUB_ERR_SCRATCH_LIMIT
    assert b"scratch" in ctypes.string_at(lib.npub_strerror(st))


def test_clearing_the_device_error_rezeroes_tile_counters(cuda_device):
    """A stream-K call whose bounded wait gave up can leave counts in its tile
    counters (the first 64 KiB of a W8A16 workspace, and of the static array
    behind npub_w8a16_gemm_noalloc, which no caller can reach).  Clearing the
    device error word (npub_device_error(1), npu.device_error(clear=True))
    re-zeroes both.  Here stale counts are written into the cached workspace
    with a fill; after the clear, both entry points give the right result."""
    from npu_comp_b200 import npu
    M, N, K = 32, 12288, 4096                      # a stream-K (decode-sized) shape
    assert "skinny" in _lib.load().npub_w8a16_kernel_name(M, N, K).decode()
    A, q, s = inputs(M, N, K, cuda_device, seed=5)
    nb.matmul(A, q, s)                             # creates the cached workspace of this stream
    key = (cuda_device.index or 0, torch.cuda.current_stream().cuda_stream)
    npu._zeroed_ws[key][: 64 << 10].fill_(0x7F)    # stale counts, as an aborted call leaves them
    assert npu.device_error(clear=True) == 0
    assert int(npu._zeroed_ws[key][: 64 << 10].count_nonzero()) == 0
    A2, q2, s2 = inputs(M, N, K, cuda_device, seed=6)
    expect = (A2.float() @ q2.float().t()) * s2.float()[None, :]
    got = nb.matmul(A2, q2, s2).float()
    assert ((got - expect).abs().max() / expect.abs().max()).item() <= TOL
    out = torch.empty((M, N), dtype=torch.float16, device=cuda_device)
    for _ in range(2):
        assert noalloc(A2, q2, s2, out) == 0
        torch.cuda.synchronize()
        assert torch.equal(out.float(), got)

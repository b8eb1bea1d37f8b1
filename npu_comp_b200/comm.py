"""Tensor-parallel all-reduce over NVLink peer memory (npub_allreduce_f16).

The reductions after the row-parallel projections of a decode step are a few
hundred KB; NCCL's per-call latency there (21 us on 2 B200s, 36 us on 8 inside
a CUDA graph) is most of a decode layer.  PeerAllReduce maps every rank's
staging buffer through CUDA IPC (handles exchanged with torch.distributed) and
reduces with one libnpub kernel per call; larger messages go to NCCL.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib


class PeerAllReduce:
    """One per (process group, device); all ranks create it together."""

    def __init__(self, group, device, max_bytes: int = 1 << 20):
        import torch.distributed as dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.max_bytes = max_bytes
        self.device = device
        lib = _lib.load()
        hb = int(lib.npub_comm_handle_bytes())
        comm = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * hb)()
        st = lib.npub_comm_create(self.world, self.rank, max_bytes, ctypes.byref(comm), handle)
        if st != _lib.NPUB_OK:
            raise _lib.NpubError("npub_comm_create", st, lib.npub_strerror(st).decode())
        self._comm = comm
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=device)
        allh = torch.empty(self.world * hb, dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(allh, mine, group=group)
        blob = bytes(allh.cpu().tolist())
        _lib.call("npub_comm_open", self._comm, blob)
        dist.barrier(group=group)

    def fits(self, t: torch.Tensor) -> bool:
        return (t.is_cuda and t.dtype == torch.float16 and t.is_contiguous() and t.numel() % 8 == 0
                and t.numel() * 2 <= self.max_bytes and t.data_ptr() % 16 == 0)

    def all_reduce_(self, t: torch.Tensor) -> None:
        """In-place sum over the ranks (t must satisfy fits())."""
        _lib.call("npub_allreduce_f16", self._comm, t.data_ptr(), t.data_ptr(), t.numel(),
                  torch.cuda.current_stream(t.device).cuda_stream)

    def all_reduce_rms(self, t: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor, out: torch.Tensor,
                       g_out: torch.Tensor, ss_out: torch.Tensor) -> None:
        """out = fp16(sum over ranks of t) + residual, g_out = fp16(out * gamma),
        ss_out [d/32, rows] the sums of out^2 per 32 columns (t: [rows, d])."""
        rows, d = t.shape
        for x in (residual, out, g_out):
            assert x.shape == t.shape and x.is_contiguous() and x.dtype == torch.float16
        _lib.call("npub_allreduce_f16_rms", self._comm, t.data_ptr(), out.data_ptr(), rows, d, residual.data_ptr(),
                  gamma.data_ptr(), g_out.data_ptr(), ss_out.data_ptr(), ss_out.stride(0),
                  torch.cuda.current_stream(t.device).cuda_stream)

    def close(self) -> None:
        if self._comm:
            _lib.load().npub_comm_destroy(self._comm)
            self._comm = None


def enabled() -> bool:
    return os.environ.get("NPUB_PEER_ALLREDUCE", "1") != "0"

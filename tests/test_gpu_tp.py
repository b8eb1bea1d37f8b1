"""Tensor-parallel Llama layer on 2 GPUs (NCCL) against the 1-GPU layer.

Each rank builds its shard of the same seeded layer (llama.make_layer with
TP(rank, 2)), runs prefill and a decode step, and rank 0 compares with the
unsharded layer run on its GPU.  Skipped when fewer than 2 GPUs are visible.
Tolerance: normwise relative error <= 1e-2 (the all-reduce sums fp16 partials
in a different order than the single-GPU accumulation)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    from npu_comp_b200 import llama
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        cfg = llama.LlamaConfig(d=1024, heads=8, kv_heads=4, head_dim=128, ffn=2752, eps=1e-5)
        tp = llama.TP(rank, world, dist.group.WORLD)
        w = llama.make_layer(cfg, seed=11, device=dev, tp=tp)
        g = torch.Generator(device=dev).manual_seed(3)
        B, T = 2, 192
        x = torch.randn((B * T, cfg.d), generator=g, device=dev).half()
        hk = cfg.kv_heads // world
        kc = torch.zeros((B, hk, 256, cfg.head_dim), dtype=torch.float16, device=dev)
        vc = torch.zeros_like(kc)
        y = llama.layer_prefill(x, w, cfg, batch=B, tp=tp, kv_out=(kc, vc))
        xd = torch.randn((B, cfg.d), generator=g, device=dev).half()
        pos = torch.full((B,), T, dtype=torch.int32, device=dev)
        yd = llama.layer_decode(xd, w, cfg, kc, vc, pos, ctx_max=T + 1, tp=tp)
        torch.cuda.synchronize()
        if rank == 0:
            w1 = llama.make_layer(cfg, seed=11, device=dev)
            kc1 = torch.zeros((B, cfg.kv_heads, 256, cfg.head_dim), dtype=torch.float16, device=dev)
            vc1 = torch.zeros_like(kc1)
            y1 = llama.layer_prefill(x, w1, cfg, batch=B, kv_out=(kc1, vc1))
            yd1 = llama.layer_decode(xd, w1, cfg, kc1, vc1, pos, ctx_max=T + 1)
            e = ((y.float() - y1.float()).abs().max() / y1.float().abs().max()).item()
            ed = ((yd.float() - yd1.float()).abs().max() / yd1.float().abs().max()).item()
            q.put((e, ed))
        dist.barrier()
        tp.close()
    finally:
        dist.destroy_process_group()


def test_tp2_layer_matches_single_gpu():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    e, ed = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert e <= TOL, e
    assert ed <= TOL, ed


def _ar_worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    from npu_comp_b200 import comm
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        peer = comm.PeerAllReduce(dist.group.WORLD, dev, max_bytes=1 << 20)
        errs, same = [], []
        sizes = [32 * 4096, 8, 4096 * 64, 1000 * 8, 32 * 4096, (1 << 20) // 2]
        for i, n in enumerate(sizes * 2):
            g = torch.Generator(device=dev).manual_seed(1000 * i + rank)
            x = torch.randn(n, generator=g, device=dev).half()
            allx = [torch.empty_like(x) for _ in range(world)]
            dist.all_gather(allx, x)
            ref = torch.stack([a.float() for a in allx]).sum(0)
            peer.all_reduce_(x)
            errs.append(((x.float() - ref).abs().max() / ref.abs().max()).item())
            got = [torch.empty_like(x) for _ in range(world)]
            dist.all_gather(got, x)
            same.append(all(torch.equal(got[0], o) for o in got))
        # replayed from a CUDA graph: the per-block epochs advance on the device
        x = torch.ones(32 * 4096, device=dev, dtype=torch.float16) * (rank + 1)
        y = x.clone()
        gr = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(gr, stream=s):
                y.copy_(x)
                peer.all_reduce_(y)
        torch.cuda.synchronize()
        graph_ok = True
        for _ in range(5):
            gr.replay()
            torch.cuda.synchronize()
            graph_ok &= bool((y.float() == world * (world + 1) / 2).all())
        del gr
        torch.cuda.synchronize()
        dist.barrier()
        peer.close()
        if rank == 0:
            q.put((max(errs), all(same), graph_ok))
    finally:
        dist.destroy_process_group()


def test_peer_allreduce_2gpu():
    """npub_allreduce_f16 on 2 GPUs: the fp32 sum within fp16 rounding, the same
    bits on every rank, across message sizes and from a replayed CUDA graph."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ar_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    err, same, graph_ok = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert err <= 1e-3, err
    assert same
    assert graph_ok


def _gemm_ar_worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    from npu_comp_b200 import comm
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NPUB_FUSED_GEMM_ALLREDUCE="1")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        peer = comm.PeerAllReduce(dist.group.WORLD, dev)
        errs, same = [], []
        shapes = [(32, 4096, 2048), (64, 4096, 5504), (5, 300, 1024), (32, 8192, 512)]
        for i, (M, N, K) in enumerate(shapes * 2):
            g = torch.Generator(device=dev).manual_seed(100 * i + rank)          # this rank's K slice
            gs = torch.Generator(device=dev).manual_seed(100 * i + 77)           # shared by the ranks
            A = torch.randn((M, K), generator=g, device=dev).half()
            W = torch.randint(-127, 128, (N, K), generator=g, device=dev, dtype=torch.int8)
            s = (torch.rand(N, generator=gs, device=dev) * 1e-3 + 1e-3).half()
            R = torch.randn((M, N), generator=gs, device=dev).half()
            allA = [torch.empty_like(A) for _ in range(world)]
            allW = [torch.empty_like(W) for _ in range(world)]
            dist.all_gather(allA, A)
            dist.all_gather(allW, W)
            ref = sum(a.float() @ w.float().t() for a, w in zip(allA, allW)) * s.float()[None, :] * 0.5 + R.float()
            out = torch.empty((M, N), dtype=torch.float16, device=dev)
            peer.matmul_allreduce(A, W, s, out=out, residual=R, alpha=0.5)
            errs.append(((out.float() - ref).abs().max() / ref.abs().max()).item())
            got = [torch.empty_like(out) for _ in range(world)]
            dist.all_gather(got, out)
            same.append(all(torch.equal(got[0], o) for o in got))
        # from a replayed CUDA graph
        M, N, K = 32, 4096, 1024
        g = torch.Generator(device=dev).manual_seed(rank)
        A = torch.randn((M, K), generator=g, device=dev).half()
        W = torch.randint(-127, 128, (N, K), generator=g, device=dev, dtype=torch.int8)
        s = torch.full((N,), 1e-3, dtype=torch.float16, device=dev)
        out = torch.empty((M, N), dtype=torch.float16, device=dev)
        peer.matmul_allreduce(A, W, s, out=out)
        first = out.clone()
        gr = torch.cuda.CUDAGraph()
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            with torch.cuda.graph(gr, stream=st):
                peer.matmul_allreduce(A, W, s, out=out)
        torch.cuda.synchronize()
        graph_ok = True
        for _ in range(4):
            out.zero_()
            gr.replay()
            torch.cuda.synchronize()
            graph_ok &= torch.equal(out, first)
        del gr
        torch.cuda.synchronize()
        dist.barrier()
        peer.close()
        if rank == 0:
            q.put((max(errs), all(same), graph_ok))
    finally:
        dist.destroy_process_group()


def test_fused_gemm_allreduce_2gpu():
    """npub_w8a16_gemm_allreduce on 2 GPUs (each rank a K slice): the fp32
    reference within TOL, the same bits on every rank, and from a graph."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gemm_ar_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    err, same, graph_ok = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert err <= TOL, err
    assert same
    assert graph_ok

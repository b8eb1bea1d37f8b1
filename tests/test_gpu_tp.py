"""Tensor-parallel Llama layer on 2, 4 and 8 GPUs (NCCL + peer all-reduce)
against the 1-GPU layer and the float64 oracle, the peer all-reduce on 2
GPUs, and a bounded wait on a peer that gives up.

Each rank builds its shard of the same seeded layer (llama.make_layer with
TP(rank, world)), runs a prefill of 2 prompts and a decode step, and rank 0
compares with the unsharded layer on its GPU and with oracle/ref.py's
ref_layer_q (model.py:115-157 in float64 on the same quantised weights).
Skipped when fewer GPUs are visible than a test needs.  NVLS is off
(NCCL_NVLS_ENABLE=0): the peer kernels use plain loads and stores.
Tolerance: normwise relative error <= 1e-2 (the all-reduce sums fp16
partials in a different order than the single-GPU accumulation)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, extra_env=None):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0", **(extra_env or {}))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    return dev


def _run(target, world, timeout=600):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = q.get(timeout=timeout)
    finally:
        for p in procs:
            p.join(timeout=120)
    for p in procs:
        assert p.exitcode == 0
    return res


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from npu_comp_b200 import llama
    from oracle import ref
    dev = _init(rank, world, port)
    try:
        cfg = llama.LlamaConfig(d=1024, heads=8, kv_heads=8, head_dim=128, ffn=2816, eps=1e-5)
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
            # the float64 oracle on the unsharded quantised weights: prompt rows, and the
            # decode token as row T of the prompt followed by that token
            L = ref.prepare_layer({n: getattr(w1, n).cpu().numpy() for n in
                                   ("wqkv", "sqkv", "wo", "so", "wgu", "sgu", "wd", "sd", "g1", "g2")})
            xh, xdh = x.float().cpu().numpy().reshape(B, T, cfg.d), xd.float().cpu().numpy()
            yo = [ref.ref_layer_q(L, np.concatenate([xh[b], xdh[b:b + 1]]), cfg.heads, cfg.kv_heads,
                                  cfg.head_dim, cfg.eps, cfg.theta) for b in range(B)]
            eo = ref.rel_err(y.float().cpu().numpy(), np.concatenate([o[:T] for o in yo]))
            edo = ref.rel_err(yd.float().cpu().numpy(), np.stack([o[T] for o in yo]))
            q.put((e, ed, eo, edo))
        dist.barrier()
        tp.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_layer_matches_single_gpu_and_oracle(world):
    e, ed, eo, edo = _run(_worker, world)
    assert e <= TOL, e
    assert ed <= TOL, ed
    assert eo <= TOL, eo
    assert edo <= TOL, edo


def _ar_worker(rank, world, port, q):
    import torch.distributed as dist
    from npu_comp_b200 import comm
    dev = _init(rank, world, port)
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
    err, same, graph_ok = _run(_ar_worker, 2, timeout=300)
    assert err <= 1e-3, err
    assert same
    assert graph_ok


def _timeout_worker(rank, world, port, q):
    import torch.distributed as dist
    dev = _init(rank, world, port, {"NPUB_WAIT_LIMIT_MS": "50"})
    from npu_comp_b200 import comm, npu
    try:
        peer = comm.PeerAllReduce(dist.group.WORLD, dev, max_bytes=1 << 20)
        n = 32 * 4096
        mk = lambda step: torch.full((n,), float(10 * step + rank + 1), device=dev, dtype=torch.float16)  # noqa: E731
        # 1. an ordinary call
        x = mk(1)
        peer.all_reduce_(x)
        torch.cuda.synchronize()
        ok1 = bool((x.float() == 11 + 12).all())
        dist.barrier()
        # 2. rank 1 skips a call: rank 0's wait for its flags gives up after 50 ms,
        #    the kernel leaves its output alone and sets the device error word
        err0 = 0
        x = mk(2)
        if rank == 0:
            peer.all_reduce_(x)
            torch.cuda.synchronize()
            err0 = npu.device_error(clear=True)
            untouched = bool((x.float() == 21).all())
        dist.barrier()
        # 3. rank 1 makes the call late: rank 0's flags and staged data are there,
        #    so it completes at once (the sum of both ranks' step-2 inputs) and the
        #    per-block epochs of the two ranks are in step again
        if rank == 1:
            peer.all_reduce_(x)
            torch.cuda.synchronize()
            late = bool((x.float() == 21 + 22).all())
        dist.barrier()
        # 4. both GPUs keep working: ordinary calls give the right sums, no error is left
        x = mk(3)
        peer.all_reduce_(x)
        torch.cuda.synchronize()
        ok4 = bool((x.float() == 31 + 32).all()) and npu.device_error() == 0
        y = torch.randn(1024, device=dev) @ torch.randn(1024, device=dev)
        ok4 &= bool(torch.isfinite(y))
        res = torch.tensor([int(ok1), err0, int(ok4), int(untouched if rank == 0 else late)], device=dev)
        allr = [torch.empty_like(res) for _ in range(world)]
        dist.all_gather(allr, res)
        dist.barrier()
        peer.close()
        if rank == 0:
            q.put([r.cpu().tolist() for r in allr])
    finally:
        dist.destroy_process_group()


def test_peer_wait_gives_up_and_both_gpus_stay_usable():
    """A bounded device wait on a peer that never arrives (rank 1 skips one
    npub_allreduce_f16 call; NPUB_WAIT_LIMIT_MS=50): rank 0's kernel returns,
    npub_device_error reports it (0x501), and both GPUs keep computing."""
    r0, r1 = _run(_timeout_worker, 2, timeout=300)
    assert r0[0] == 1 and r1[0] == 1
    assert r0[1] == 0x501, hex(r0[1])      # NPUB_ERR_DEVICE_TIMEOUT cause: peer flag wait (comm.cu)
    assert r0[3] == 1                      # rank 0's output was left as it was
    assert r1[3] == 1                      # the late call completed with both ranks' data
    assert r0[2] == 1 and r1[2] == 1


def _ar_rms_worker(rank, world, port, q):
    import torch.distributed as dist
    dev = _init(rank, world, port)
    from npu_comp_b200 import comm
    try:
        peer = comm.PeerAllReduce(dist.group.WORLD, dev, max_bytes=1 << 20)
        g = torch.Generator(device=dev).manual_seed(11)   # the same residual / gamma on every rank
        rows, d = 32, 4096
        res = torch.randn((rows, d), generator=g, device=dev).half()
        gam = (1 + 0.1 * torch.randn(d, generator=g, device=dev)).half()
        gr = torch.Generator(device=dev).manual_seed(100 + rank)
        part = torch.randn((rows, d), generator=gr, device=dev).half()
        out, G = torch.empty_like(part), torch.empty_like(part)
        ss = torch.empty((d // 32, rows), dtype=torch.float32, device=dev)
        peer.all_reduce_rms(part, res, gam, out, G, ss)
        # the plain all-reduce of the same partials, then the residual add in torch
        s = part.clone()
        peer.all_reduce_(s)
        torch.cuda.synchronize()
        want = (s.float() + res.float()).half()
        ok_out = torch.equal(out, want)
        ok_g = torch.equal(G, (out.float() * gam.float()).half())
        ssr = (out.double() ** 2).view(rows, d // 32, 32).sum(-1).t()
        ss_err = ((ss.double() - ssr).abs().max() / ssr.abs().max()).item()
        allo = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(allo, out)
        same = all(torch.equal(allo[0], o) for o in allo)
        dist.barrier()
        peer.close()
        if rank == 0:
            q.put((ok_out, ok_g, ss_err, same))
    finally:
        dist.destroy_process_group()


def test_peer_allreduce_rms_2gpu():
    """npub_allreduce_f16_rms on 2 GPUs: out = fp16(sum) + residual bit for bit
    against the plain all-reduce and a torch add, G = fp16(out * gamma) bit for
    bit, the per-32-column sums of out^2, the same bits on every rank."""
    ok_out, ok_g, ss_err, same = _run(_ar_rms_worker, 2, timeout=300)
    assert ok_out and ok_g and same
    assert ss_err <= 1e-5, ss_err

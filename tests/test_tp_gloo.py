"""Tensor-parallel decomposition of the Llama layer on CPU ranks (gloo).

Each of 2 (or 4) ranks takes its shards with llama.tp_ranges (the same slicing the
GPU layer uses), computes its partial layer in float64 torch, and the
row-parallel partials are summed with TP.all_reduce over a gloo process
group.  The result must equal the unsharded layer."""
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from npu_comp_b200 import llama

CFG = llama.LlamaConfig(d=64, heads=4, kv_heads=2, head_dim=16, ffn=96, eps=1e-5, theta=10000.0, vocab=64, layers=1)
# grouped heads that split over 4 ranks (2 query heads and 1 kv head per rank)
CFG4 = llama.LlamaConfig(d=64, heads=8, kv_heads=4, head_dim=8, ffn=128, eps=1e-5, theta=10000.0, vocab=64,
                         layers=1)


def weights(seed=0, c=CFG):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64) * 0.1  # noqa: E731
    return {"qkv": r(c.d, c.q_dim + 2 * c.kv_dim), "o": r(c.q_dim, c.d), "gu": r(c.d, 2 * c.ffn), "d": r(c.ffn, c.d),
            "g1": 1 + 0.1 * r(c.d), "g2": 1 + 0.1 * r(c.d)}


def rope(x, heads, hd, T, theta=CFG.theta):
    half = hd // 2
    f = theta ** (-2.0 * torch.arange(half, dtype=torch.float64) / hd)
    ang = torch.arange(T, dtype=torch.float64)[:, None] * f[None]
    c, s = torch.cos(ang), torch.sin(ang)
    x = x.view(T, heads, hd)
    a, b = x[..., :half], x[..., half:]
    return torch.cat([a * c[:, None] - b * s[:, None], b * c[:, None] + a * s[:, None]], -1).reshape(T, heads * hd)


def partial_layer(x, W, rank, size, tp, c=CFG):
    """This rank's part of the layer; all_reduce completes the row-parallel sums."""
    T = x.shape[0]
    rg = llama.tp_ranges(c, rank, size)
    hq, hk, hd = c.heads // size, c.kv_heads // size, c.head_dim
    rms = lambda v, g: v / torch.sqrt((v * v).mean(1, keepdim=True) + c.eps) * g  # noqa: E731
    cols = torch.cat([torch.arange(r.start, r.stop) for r in rg["qkv"]])
    qkv = rms(x, W["g1"]) @ W["qkv"][:, cols]
    q = rope(qkv[:, :hq * hd], hq, hd, T, c.theta)
    k = rope(qkv[:, hq * hd:(hq + hk) * hd], hk, hd, T, c.theta)
    v = qkv[:, (hq + hk) * hd:]
    ctx = torch.zeros(T, hq * hd, dtype=torch.float64)
    mask = torch.triu(torch.ones(T, T, dtype=torch.bool), 1)
    for h in range(hq):
        kv = h // (hq // hk)
        S = (q[:, h * hd:(h + 1) * hd] @ k[:, kv * hd:(kv + 1) * hd].T) / math.sqrt(hd)
        P = torch.softmax(S.masked_fill(mask, float("-inf")), -1)
        ctx[:, h * hd:(h + 1) * hd] = P @ v[:, kv * hd:(kv + 1) * hd]
    o = rg["o"][0]
    h_part = ctx @ W["o"][o.start:o.stop]
    tp.all_reduce(h_part)
    h_part = h_part + x                # residual after the reduction (as the GPU layer does)
    cols = torch.cat([torch.arange(r.start, r.stop) for r in rg["gu"]])
    gu = rms(h_part, W["g2"]) @ W["gu"][:, cols]
    f = c.ffn // size
    a = gu[:, :f] / (1 + torch.exp(-gu[:, :f])) * gu[:, f:]
    dr = rg["d"][0]
    y = a @ W["d"][dr.start:dr.stop]
    tp.all_reduce(y)
    return y + h_part


def _worker(rank, size, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=size)
    try:
        c = CFG if size <= 2 else CFG4
        x = torch.randn(12, c.d, generator=torch.Generator().manual_seed(5), dtype=torch.float64)
        y = partial_layer(x, weights(c=c), rank, size, llama.TP(rank, size, dist.group.WORLD), c)
        q.put((rank, y))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("size", [2, 4])
def test_tp_equals_single_rank(size):
    c = CFG if size <= 2 else CFG4
    x = torch.randn(12, c.d, generator=torch.Generator().manual_seed(5), dtype=torch.float64)
    ref = partial_layer(x, weights(c=c), 0, 1, llama.TP(), c)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, size, port, q)) for r in range(size)]
    for p in procs:
        p.start()
    outs = dict(q.get(timeout=120) for _ in range(size))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(size):
        assert torch.allclose(outs[r], ref, rtol=1e-10, atol=1e-10)


def test_tp_ranges_partition_the_weights():
    for c, size in ((CFG, 1), (CFG, 2), (CFG4, 4), (llama.LLAMA_7B, 8)):
        seen = {k: [] for k in ("qkv", "o", "gu", "d")}
        for r in range(size):
            for k, v in llama.tp_ranges(c, r, size).items():
                for rg in v:
                    seen[k].extend(rg)
        assert sorted(seen["qkv"]) == list(range(c.q_dim + 2 * c.kv_dim))
        assert sorted(seen["o"]) == list(range(c.q_dim))
        assert sorted(seen["gu"]) == list(range(2 * c.ffn))
        assert sorted(seen["d"]) == list(range(c.ffn))
    with pytest.raises(ValueError):
        llama.tp_ranges(CFG, 0, 3)
    # Llama-7B shapes at 8 ranks: 11008/8 = 1376 is a multiple of 16 (the GEMM's K granularity)
    rg = llama.tp_ranges(llama.LLAMA_7B, 7, 8)
    assert len(rg["d"][0]) == 1376 and 1376 % 16 == 0


def test_flop_and_byte_counts():
    c = llama.LLAMA_7B
    assert c.linear_flops_per_token() == 2 * 4096 * (12288 + 4096 + 22016 + 11008)
    assert abs(llama.layer_flops(c, 2048, 2048) - 863.3e9) / 863.3e9 < 1e-3
    assert abs(llama.decode_bytes(c, 64, 4096) - 4.5e9) / 4.5e9 < 0.01


@pytest.mark.parametrize("size", [1, 2])
def test_gate_up_interleave_after_sharding(size):
    """The layer's gate|up weights: each rank slices its F/TP gate and up rows
    (tp_ranges) and interleaves them, row 2c = gate channel c, 2c + 1 = up
    channel c of that rank, scales alike (the layout the SwiGLU epilogue reads
    from adjacent lanes)."""
    from npu_comp_b200 import npu
    F = CFG.ffn
    rows = torch.arange(2 * F, dtype=torch.int32)  # row r of the full [gate | up] matrix
    q = rows[:, None].repeat(1, 16).to(torch.int8 if 2 * F < 128 else torch.int32)
    s = rows.to(torch.float16)
    for rank in range(size):
        rg = llama.tp_ranges(CFG, rank, size)["gu"]
        idx = torch.cat([torch.arange(r.start, r.stop) for r in rg])
        qi, si = npu.interleave_gate_up(q.index_select(0, idx).contiguous(), s.index_select(0, idx).contiguous())
        f = F // size
        for c in range(f):
            assert int(qi[2 * c, 0]) == rank * f + c and int(qi[2 * c + 1, 0]) == F + rank * f + c
            assert float(si[2 * c]) == rank * f + c and float(si[2 * c + 1]) == F + rank * f + c
        assert bool((qi == qi[:, :1]).all())  # whole rows moved

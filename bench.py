"""Benchmark of the W8A16 / Llama-layer hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload stack|layer|decode|gemm]

Default workload ("stack"): the 32-layer Llama-7B-shaped decoder (d 4096,
32 heads x 128, FFN 11008, vocab 32000 fp16 lm_head, RoPE theta 10000), all
seven linears of every layer W8A16 (int8 weights ~N(0, 0.02) quantised per
output channel), random-init weights, 32 seeded prompts x 1024 tokens of
prefill followed by 128 greedy decode steps.  A step is one prefill plus the
128 decode steps; the metric is (prompt + generated) tokens per second.  With
--gpus N under torchrun the stack runs tensor-parallel over N GPUs (NCCL
all-reduces after the row-parallel projections; total work fixed: strong
scaling).

Other workloads: "layer" (one layer, prefill of a 2048-token prompt),
"decode" (one layer, 64 sequences x 1 token over a 4096-token KV cache),
"gemm" (the layer's gate|up W8A16 GEMM, 2048 x 22016 x 4096).

Rank 0 prints one JSON line.  `roofline` covers the dominant kernel, the
tcgen05 W8A16 GEMM, timed with CUDA events on its launch stream.
`cpu_baseline` is the reference cmodel (mysim, built from the reference's
_poc/mysim.cpp) or its C restatement, run on a bounded sample of the
workload's GEMMs on this host's cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

HERE = os.path.dirname(os.path.abspath(__file__))
METRIC = "W8A16 GEMM TFLOP/s + Llama-layer tokens/s, % of roofline, 1/2/4/8 B200 vs mysim"
L2_BYTES = 126 * 1024 * 1024


def _peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), \
            "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


def _traffic(key):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    try:
        with open(os.path.join(HERE, "profiles", "traffic.json")) as f:
            return json.load(f).get(key)
    except Exception:
        return None


class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.t0 = time.time()
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first_sample(self, timeout=3.0):
        """Block until nvidia-smi has produced a sample (its start-up takes ~0.5 s)."""
        t0 = time.time()
        while self.proc is not None and not self.lines and time.time() - t0 < timeout:
            time.sleep(0.02)
        self.lines.clear()

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 6:
                continue
            try:
                sm.append(float(parts[0]))
                mx = max(mx, float(parts[1]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[2:6]):
                if v.lower() in ("active", "1", "0x1"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- CPU baselines
#
# Two CPU paths are timed on this host, as the reference's own numbers would be:
#  * mysim, the reference's cmodel (built from its _poc/mysim.cpp into
#    oracle/_ref/mysim; the C restatement of it when absent), driven like the
#    reference's run() (npu.py:62-71) on the programs the reference emits for
#    each op: the 64-tiled W8A16 matmul (codegen.py:59-108) and the RMSNorm,
#    SwiGLU, masked-softmax and RoPE recipes (test_rmsnorm.py, test_swiglu.py,
#    test_attention.py, llama_layer.py:96-104).  Each program is run on a
#    bounded sample; the workload's time is projected from the measured rate
#    of each op kind (FLOPs or elements per second) times the workload's
#    count of that kind.  mysim is single-threaded: `cores` processes run
#    concurrently for the multi-core figure.
#  * PyTorch on the CPU: fp32 compute on the same fp16 / int8 synthetic
#    tensors (weights dequantised to fp32 once), all host threads.

def _cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def _mysim_program(kind):
    """(words, G-buffer image, gn, work units of one run, unit) for one op kind."""
    import numpy as np
    sys.path.insert(0, HERE)
    from oracle import emit, ref
    rng = np.random.default_rng(0)
    if kind == "gemm":  # 64 tokens x 512 output channels x K 4096 of the QKV projection
        M, N, K = 64, 512, 4096
        A = rng.standard_normal((M, K)).astype(np.float16)
        q, s = ref.quantize_w8((rng.standard_normal((K, N)) * 0.02).astype(np.float32))
        words, g, _, gn = emit.w8a16_program(A, ref.dequant_f16(q, s))
        return words, g, gn, 2.0 * M * N * K, "FLOP"
    if kind == "rmsnorm":
        X = rng.standard_normal((512, 248)).astype(np.float16)
        words, g, _, gn = emit.rmsnorm_program(X, np.ones(248))
        return words, g, gn, float(X.size), "elements"
    if kind == "swiglu":
        n = 1 << 18
        words, g, _, gn = emit.swiglu_program(rng.standard_normal(n).astype(np.float16),
                                              rng.standard_normal(n).astype(np.float16))
        return words, g, gn, float(n), "elements"
    if kind == "softmax":
        S = rng.standard_normal((255, 255)).astype(np.float16)
        words, g, _, gn = emit.softmax_program(S)
        return words, g, gn, float(S.size), "elements"
    if kind == "rope":
        Q = rng.standard_normal((256, 128)).astype(np.float16)
        c, s_ = ref.rope_tables(256, 128)
        words, g, _, gn = emit.rope_program(Q, ref.f16(c), ref.f16(s_))
        return words, g, gn, float(Q.size), "elements"
    raise ValueError(kind)


MYSIM_KINDS = ("gemm", "rmsnorm", "swiglu", "softmax", "rope")


def mysim_rates(kinds=MYSIM_KINDS, all_cores=False, reps=None):
    """Measured mysim rate of each op kind (units per second over all processes
    that ran at once).  Returns (rates, processes, kind, per-kind sample text)."""
    import tempfile
    import numpy as np
    sys.path.insert(0, HERE)
    from oracle import cmodel
    nproc = _cpu_cores() if all_cores else 1
    use_ref = cmodel.have_mysim()
    reps = reps or {"gemm": 1, "rmsnorm": 2, "swiglu": 2, "softmax": 8, "rope": 8}
    rates, notes = {}, []
    for kind in kinds:
        words, gimg, gn, units, uname = _mysim_program(kind)
        r = reps.get(kind, 1)
        if use_ref:
            d = tempfile.mkdtemp()
            with open(os.path.join(d, "program_memory.bin"), "wb") as f:
                f.write(np.asarray(words, dtype="<u4").tobytes() + b"\n")
            with open(os.path.join(d, "G_buffer_data.bin"), "wb") as f:
                f.write(np.asarray(gimg).astype("<f2").tobytes() + b"\n")
            cmd = " ; ".join([f"{cmodel.MYSIM} --run {len(words) + 1}"] * r)
            t0 = time.time()
            procs = [subprocess.Popen(["/bin/sh", "-c", cmd], cwd=d, stdout=subprocess.DEVNULL,
                                      stderr=subprocess.DEVNULL) for _ in range(nproc)]
            for p in procs:
                p.wait()
            dt = time.time() - t0
        else:
            from concurrent.futures import ProcessPoolExecutor
            import multiprocessing as mp
            t0 = time.time()
            with ProcessPoolExecutor(max_workers=nproc, mp_context=mp.get_context("spawn")) as ex:
                list(ex.map(_run_port, [(words, gimg, gn, r)] * nproc))
            dt = time.time() - t0
        rates[kind] = units * r * nproc / dt
        notes.append(f"{kind} {units * r:.3g} {uname} x {nproc} proc in {dt:.2f} s")
    return rates, nproc, "reference" if use_ref else "port", "; ".join(notes)


def _run_port(args):
    sys.path.insert(0, HERE)
    from oracle import cmodel
    words, gimg, gn, reps = args
    for _ in range(reps):
        cmodel.run_oracle(words, gimg, gn, maxrun=len(words) + 1)
    return 0


def workload_ops(workload, shape=None):
    """What one unit of the workload asks of the NPU program path, per op kind
    (FLOPs for the matmuls -- linears and the attention products, full T x T as
    the NPU computes them before masking -- and elements for the vector
    recipes), and the unit's name.  Units: a token (layer, decode, stack), a
    TFLOP (gemm) or a GB of the vector ops' algorithmic traffic (vector)."""
    sys.path.insert(0, HERE)
    from npu_comp_b200.llama import LLAMA_7B as c
    H, KV, hd, d, F = c.heads, c.kv_heads, c.head_dim, c.d, c.ffn
    lin = c.linear_flops_per_token()

    def per_token(T_q, ctx):  # one layer, one query token attending to ctx keys
        return {"gemm": lin + 4.0 * H * hd * ctx, "rmsnorm": 2.0 * d, "swiglu": float(F),
                "softmax": float(H * ctx), "rope": float((H + KV) * hd)}

    if workload == "gemm":
        return {"gemm": 1e12}, "TFLOP/s"
    if workload == "vector":
        b = vector_bytes()
        tot = sum(b.values()) / 1e9
        return {"rmsnorm": 2048 * 4096 / tot, "swiglu": 2048 * 11008 / tot, "softmax": 32 * 2048 * 2048 / tot}, "GB/s"
    if workload == "layer":
        return per_token(1, 2048), "tokens/s"      # every query row sees the full (masked) 2048-key row
    if workload == "decode":
        return per_token(1, 4097), "tokens/s"
    # stack: 32 prompts x 1024 prefill + 128 greedy steps, 32 layers + lm_head per generated token
    B, T, S, L = 32, 1024, 128, c.layers
    tot = {k: 0.0 for k in MYSIM_KINDS}
    for k, v in per_token(1, T).items():
        tot[k] += v * B * T * L
    for s in range(S):
        for k, v in per_token(1, T + s + 1).items():
            tot[k] += v * B * L
    tot["gemm"] += 2.0 * d * c.vocab * B * (S + 1)
    return {k: v / (B * (T + S)) for k, v in tot.items()}, "tokens/s"


def vector_bytes():
    """Algorithmic HBM bytes of the vector-op workload (2048 tokens): RMSNorm
    x read + y written (+ gamma), SwiGLU g, u read + h written, causal softmax
    of 32 x 2048 x 2048 scores: the unmasked entries read, every entry written
    (masked ones as zeros)."""
    T, d, F, H = 2048, 4096, 11008, 32
    return {"rmsnorm": 2 * T * d * 2 + d * 2, "swiglu": 3 * T * F * 2,
            "softmax": H * (T * (T + 1) // 2) * 2 + H * T * T * 2}


def vector_isolated_us(dev, gen, reps=24):
    """Device time per launch of each vector op alone: a CUDA graph of `reps`
    launches over rotating copies of its operands (together larger than L2,
    so every launch reads from HBM), timed with CUDA events."""
    import torch
    from npu_comp_b200 import npu
    T, d, F = 2048, 4096, 11008
    out = {}

    def copies(nbytes_per_set):
        return max(2, -(-2 * L2_BYTES // nbytes_per_set))

    n = copies(2 * T * d * 2)
    xs = [torch.randn((T, d), generator=gen, device=dev).half() for _ in range(n)]
    ys = [torch.empty_like(xs[0]) for _ in range(n)]
    gam = torch.ones((d,), dtype=torch.float16, device=dev)
    ops = {"rmsnorm": [lambda i=i: npu.rmsnorm(xs[i], gam, 1e-5, out=ys[i]) for i in range(n)]}
    n2 = copies(3 * T * F * 2)
    gs = [torch.randn((T, F), generator=gen, device=dev).half() for _ in range(n2)]
    us = [torch.randn((T, F), generator=gen, device=dev).half() for _ in range(n2)]
    hs = [torch.empty_like(gs[0]) for _ in range(n2)]
    ops["swiglu"] = [lambda i=i: npu.swiglu(gs[i], us[i], out=hs[i]) for i in range(n2)]
    n3 = 2
    ss = [torch.randn((32, T, T), generator=gen, device=dev).half() for _ in range(n3)]
    ps = [torch.empty_like(ss[0]) for _ in range(n3)]
    ops["softmax"] = [lambda i=i: npu.softmax(ss[i], causal=True, out=ps[i]) for i in range(n3)]
    for name, fns in ops.items():
        for f in fns:  # warm-up outside capture
            f()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for r in range(reps):
                fns[r % len(fns)]()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(3):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        out[name] = round(e0.elapsed_time(e1) * 1e3 / (3 * reps), 2)
        del g
    return out


def reference_value(workload, rates):
    """Projected units/s of the NPU program path from the measured mysim rates."""
    ops, unit = workload_ops(workload)
    sec = sum(ops[k] / rates[k] for k in ops)
    return 1.0 / sec, unit


def torch_cpu_baseline(workload, shape=None):
    """PyTorch on all host threads, fp32 compute on the workload's fp16/int8
    tensors (weights dequantised once, outside the timed region).  Returns
    {value, unit, cores, kind, sample}."""
    import torch
    import torch.nn.functional as Fn
    sys.path.insert(0, HERE)
    from npu_comp_b200.llama import LLAMA_7B as c
    cores = _cpu_cores()
    torch.set_num_threads(cores)
    g = torch.Generator().manual_seed(0)
    f16 = lambda *sh: torch.randn(*sh, generator=g).half().float()  # noqa: E731

    def deq(n, k):  # per-channel int8 weights dequantised to fp32, [n, k]
        w = torch.randn(n, k, generator=g) * 0.02
        s = (w.abs().amax(1) / 127).half().float()
        return (torch.clamp(torch.round(w / s[:, None]), -127, 127) * s[:, None]).contiguous()

    def timed(fn, reps=2):
        fn()
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        return (time.perf_counter() - t0) / reps

    def rms(x, gm):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + c.eps) * gm

    def rope(x, heads, pos):
        half = c.head_dim // 2
        inv = c.theta ** (-2.0 * torch.arange(half, dtype=torch.float64) / c.head_dim)
        ang = (pos.double()[:, None] * inv[None, :]).float()
        cs, sn = ang.cos(), ang.sin()
        x = x.view(x.shape[0], heads, c.head_dim)
        a, b = x[..., :half], x[..., half:]
        return torch.cat([a * cs[:, None] - b * sn[:, None], b * cs[:, None] + a * sn[:, None]], -1).flatten(1)

    W = None

    def layer_weights():
        nonlocal W
        if W is None:
            W = {"qkv": deq(c.q_dim + 2 * c.kv_dim, c.d), "o": deq(c.d, c.q_dim), "gu": deq(2 * c.ffn, c.d),
                 "d": deq(c.d, c.ffn), "g": torch.ones(c.d)}
        return W

    def prefill_layer(x):  # one sequence x [T, d]
        w = layer_weights()
        T = x.shape[0]
        pos = torch.arange(T)
        qkv = rms(x, w["g"]) @ w["qkv"].T
        q = rope(qkv[:, :c.q_dim], c.heads, pos).view(T, c.heads, c.head_dim).transpose(0, 1)
        k = rope(qkv[:, c.q_dim:c.q_dim + c.kv_dim], c.kv_heads, pos).view(T, c.kv_heads, c.head_dim).transpose(0, 1)
        v = qkv[:, c.q_dim + c.kv_dim:].reshape(T, c.kv_heads, c.head_dim).transpose(0, 1)
        o = Fn.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(0, 1).reshape(T, c.q_dim)
        h = x + o @ w["o"].T
        gu = rms(h, w["g"]) @ w["gu"].T
        return h + (Fn.silu(gu[:, :c.ffn]) * gu[:, c.ffn:]) @ w["d"].T

    def decode_layer(x, kc, vc, ctx):  # x [B, d]; caches [B, KV, ctx + 1, hd], position ctx is the new token
        w = layer_weights()
        B = x.shape[0]
        pos = torch.full((B,), ctx)
        qkv = rms(x, w["g"]) @ w["qkv"].T
        q = rope(qkv[:, :c.q_dim], c.heads, pos).view(B, c.heads, 1, c.head_dim)
        kc[:, :, ctx] = rope(qkv[:, c.q_dim:c.q_dim + c.kv_dim], c.kv_heads, pos).view(B, c.kv_heads, c.head_dim)
        vc[:, :, ctx] = qkv[:, c.q_dim + c.kv_dim:].view(B, c.kv_heads, c.head_dim)
        o = Fn.scaled_dot_product_attention(q, kc[:, :, :ctx + 1], vc[:, :, :ctx + 1]).reshape(B, c.q_dim)
        h = x + o @ w["o"].T
        gu = rms(h, w["g"]) @ w["gu"].T
        return h + (Fn.silu(gu[:, :c.ffn]) * gu[:, c.ffn:]) @ w["d"].T

    if workload == "gemm":
        M, N, K = shape or (2048, 2 * c.ffn, c.d)
        A, Wd = f16(M, K), deq(N, K)
        t = timed(lambda: A @ Wd.T, reps=3)
        return {"value": 2.0 * M * N * K / t / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "pytorch-cpu",
                "sample": f"fp32 {M}x{N}x{K} matmul on dequantised int8 weights, full size"}
    if workload == "vector":
        x, gm = f16(2048, 4096), f16(4096) * 0.02 + 1
        gt, ut = f16(2048, 11008), f16(2048, 11008)
        sc = f16(32, 2048, 2048)
        mask = torch.ones(2048, 2048, dtype=torch.bool).triu(1)
        ts = {"rmsnorm": timed(lambda: rms(x, gm)), "swiglu": timed(lambda: Fn.silu(gt) * ut),
              "softmax": timed(lambda: torch.softmax(sc.masked_fill(mask, float("-inf")), -1))}
        b = vector_bytes()
        return {"value": sum(b.values()) / sum(ts.values()) / 1e9, "unit": "GB/s", "cores": cores,
                "kind": "pytorch-cpu", "per_op_gbs": {k: b[k] / ts[k] / 1e9 for k in ts},
                "sample": "fp32 RMSNorm [2048,4096], SwiGLU [2048,11008], causal softmax [32,2048,2048], full size"}
    if workload == "layer":
        x = f16(2048, c.d)
        t = timed(lambda: prefill_layer(x), reps=1)
        return {"value": 2048 / t, "unit": "tokens/s", "cores": cores, "kind": "pytorch-cpu",
                "sample": "fp32 Llama-7B layer, one 2048-token prompt, full size"}
    if workload == "decode":
        B, ctx = 16, 4096
        kc, vc = f16(B, c.kv_heads, ctx + 1, c.head_dim), f16(B, c.kv_heads, ctx + 1, c.head_dim)
        x = f16(B, c.d)
        t = timed(lambda: decode_layer(x, kc, vc, ctx), reps=2)
        return {"value": B / t, "unit": "tokens/s", "cores": cores, "kind": "pytorch-cpu",
                "sample": f"fp32 Llama-7B decode layer, {B} of the 64 sequences, KV 4096"}
    # stack: one layer of one prompt's prefill and of one batch-32 decode step,
    # projected over 32 layers x (32 prompts + 128 steps) plus the lm_head
    x = f16(1024, c.d)
    t_pre = timed(lambda: prefill_layer(x), reps=1)
    B, ctx = 32, 1024 + 64
    kc, vc = f16(B, c.kv_heads, ctx + 1, c.head_dim), f16(B, c.kv_heads, ctx + 1, c.head_dim)
    xd = f16(B, c.d)
    t_dec = timed(lambda: decode_layer(xd, kc, vc, ctx), reps=2)
    lm, hl = deq(c.vocab, c.d), f16(B, c.d)
    t_lm = timed(lambda: hl @ lm.T, reps=2)
    total = c.layers * (32 * t_pre + 128 * t_dec) + 129 * t_lm
    return {"value": 32 * (1024 + 128) / total, "unit": "tokens/s", "cores": cores, "kind": "pytorch-cpu",
            "sample": f"fp32; measured one layer of a 1024-token prompt ({t_pre:.3f} s), one batch-32 decode layer "
                      f"at KV {ctx} ({t_dec:.3f} s) and the lm_head ({t_lm:.4f} s); projected over 32 layers x "
                      "(32 prompts + 128 steps)"}


# ---------------------------------------------------------------- our arm

def setup_dist(n_gpus):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    if n_gpus > 1 or "RANK" in os.environ:
        rank = int(os.environ.get("RANK", 0))
        world = int(os.environ.get("WORLD_SIZE", 1))
        local = int(os.environ.get("LOCAL_RANK", rank))
        torch.cuda.set_device(local)
        if world > 1:
            dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
        return rank, world, local
    torch.cuda.set_device(0)
    return 0, 1, 0


def run_ours(args):
    import torch
    sys.path.insert(0, HERE)
    from npu_comp_b200 import llama, npu, _lib
    rank, world, local = setup_dist(args.gpus)
    dev = torch.device("cuda", local)
    import torch.distributed as dist
    group = dist.group.WORLD if world > 1 else None
    tp = llama.TP(rank, world, group)
    cfg = llama.LLAMA_7B
    hbm, tf_burst, tf_sust, peak_src = _peaks()

    wl = args.workload
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234)
    if wl == "layer":
        T = 2048
        w = llama.make_layer(cfg, seed=0, device=dev, tp=tp)
        x = torch.randn((T, cfg.d), generator=gen, device=dev).half()
        sc = llama.Scratch()
        y = torch.empty_like(x)
        step = lambda ev=None: llama.layer_prefill(x, w, cfg, tp=tp, scratch=sc, out=y, events=ev)  # noqa: E731
        units = float(T)
        unit = "tokens/s"
        config = {"workload": "llama7b_layer_prefill_w8a16", "tokens": T, "batch": 1, "d": cfg.d,
                  "heads": cfg.heads, "head_dim": cfg.head_dim, "ffn": cfg.ffn, "theta": cfg.theta,
                  "parallelism": f"tp{world}", "l2": "inputs larger than L2 (202 MB int8 weights per step)"}
        h_in, d_out = x, y
    elif wl == "decode":
        B, ctx = args.batch or 64, args.ctx or 4096
        w = llama.make_layer(cfg, seed=0, device=dev, tp=tp)
        hk = cfg.kv_heads // world
        kc = torch.randn((B, hk, ctx + 8, cfg.head_dim), generator=gen, device=dev).half()
        vc = torch.randn((B, hk, ctx + 8, cfg.head_dim), generator=gen, device=dev).half()
        x = torch.randn((B, cfg.d), generator=gen, device=dev).half()
        pos = torch.full((B,), ctx, dtype=torch.int32, device=dev)
        sc = llama.Scratch()
        y = torch.empty_like(x)
        step = lambda ev=None: llama.layer_decode(x, w, cfg, kc, vc, pos, ctx_max=ctx + 1, tp=tp,  # noqa: E731
                                                  scratch=sc, out=y, events=ev)
        units = float(B)
        unit = "tokens/s"
        config = {"workload": "llama7b_layer_decode_w8a16", "batch": B, "kv_len": ctx, "parallelism": f"tp{world}",
                  "l2": "inputs larger than L2 (4.3 GB KV cache per step)"}
        h_in, d_out = x, y
    elif wl == "vector":
        # RMSNorm [2048, 4096], SwiGLU [2048, 11008], causal row softmax [32, 2048, 2048]
        x = torch.randn((2048, cfg.d), generator=gen, device=dev).half()
        gam = (1 + 0.02 * torch.randn((cfg.d,), generator=gen, device=dev)).half()
        gt = torch.randn((2048, cfg.ffn), generator=gen, device=dev).half()
        ut = torch.randn((2048, cfg.ffn), generator=gen, device=dev).half()
        sc_in = torch.randn((32, 2048, 2048), generator=gen, device=dev).half()
        y = torch.empty_like(x)
        h = torch.empty_like(gt)
        pr = torch.empty_like(sc_in)
        vb = vector_bytes()

        def step(ev=None):
            mk = llama._Marks(ev)
            mk("rmsnorm")
            npu.rmsnorm(x, gam, 1e-5, out=y)
            mk("swiglu")
            npu.swiglu(gt, ut, out=h)
            mk("softmax")
            npu.softmax(sc_in, causal=True, out=pr)
            mk.end()
        units = sum(vb.values()) / 1e9
        unit = "GB/s"
        config = {"workload": "llama_vector_ops_prefill"}
        h_in, d_out = [x, gt, ut, sc_in], [y, h, pr]
    else:  # gemm: the layer's gate|up projection alone (or --shape M,N,K)
        M, N, K = (2048, 2 * cfg.ffn // world, cfg.d) if not args.shape else map(int, args.shape.split(","))
        Wf = torch.randn((K, N), generator=gen, device=dev) * 0.02
        q, s = npu.quantize_w8(Wf)
        del Wf
        A = torch.randn((M, K), generator=gen, device=dev).half()
        C = torch.empty((M, N), dtype=torch.float16, device=dev)
        step = lambda: npu.matmul(A, q, s, out=C)  # noqa: E731
        units = 2.0 * M * N * K / 1e12
        unit = "TFLOP/s"
        config = {"workload": "w8a16_gemm", "M": M, "N": N, "K": K, "parallelism": f"replica{world}",
                  "l2": "flushed: 256 MB buffer written between steps"}
        h_in, d_out = A, C

    flush = None
    if wl == "gemm":
        flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
        if flush is not None:
            flush.fill_(1.0)
    torch.cuda.synchronize()
    barrier()

    # The step is replayed from a CUDA graph: one launch per step instead of
    # ~15 host-side op calls (the kernels and their arguments are identical).
    eager_step = step
    graph = None
    if not args.eager and world == 1:
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                eager_step()
            torch.cuda.synchronize()
            step = graph.replay
            for _ in range(2):
                step()
            torch.cuda.synchronize()
        except Exception as e:  # keep the eager step (the line says which)
            print(f"graph capture failed, timing eager launches: {e}", file=sys.stderr)
            graph = None
            step = eager_step

    # ---- timed region (device time, CUDA events, max over ranks)
    c0 = _lib.launch_count()
    eager_step()
    torch.cuda.synchronize()
    launches_per_step = _lib.launch_count() - c0  # kernels of one step (a graph replay bypasses the counter)
    if args.steps is None:
        # no --steps: enough steps for ~0.6 s of timed work (the clock sampler
        # needs a few 50 ms samples), the same count on every rank
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(5):
            if flush is not None:
                flush.fill_(1.0)
            step()
        e1.record()
        torch.cuda.synchronize()
        est = torch.tensor([e0.elapsed_time(e1) / 5], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(est, op=dist.ReduceOp.MAX)
        args.steps = int(min(20000, max(50, 600.0 / max(float(est.item()), 1e-3))))
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    try:
        smi_id = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        smi_id = local
    with ClockSampler(smi_id) as clk:
        clk.wait_first_sample()
        torch.cuda.synchronize()
        barrier()
        for i in range(args.steps):
            if flush is not None:
                flush.fill_(1.0)
            ev[i][0].record()
            step()
            ev[i][1].record()
        torch.cuda.synchronize()
        barrier()
    launches = launches_per_step * args.steps
    step_ms = sum(a.elapsed_time(b) for a, b in ev)
    t = torch.tensor([step_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms = float(t.item())
    ms_per_step = step_ms / args.steps
    per_rank_units = units  # TP: every rank processes the same tokens (strong scaling)
    replicas = wl in ("gemm", "vector")  # independent copies per GPU: weak scaling
    value = per_rank_units / (ms_per_step / 1e3) if not replicas else units * world / (ms_per_step / 1e3)

    # Dominant kernel roofline and per-op breakdown: eager steps with CUDA events
    # around each op on its stream, each enqueued behind a graph replay so that the
    # host is ahead of the device and the events bracket device time only.
    reps = max(1, min(args.steps, 10))
    npu.gemm_events = []
    evs = [] if wl in ("layer", "decode", "vector") else None
    for _ in range(reps):
        if flush is not None:
            flush.fill_(1.0)
        if graph is not None:
            graph.replay()
        eager_step(evs) if evs is not None else eager_step()
    torch.cuda.synchronize()
    gev = npu.gemm_events
    npu.gemm_events = None
    breakdown = None
    if evs is not None:
        breakdown = {}
        for name, a_, b_ in evs:
            breakdown[name] = breakdown.get(name, 0.0) + a_.elapsed_time(b_) * 1e3 / reps
        breakdown = {k_: round(v_, 1) for k_, v_ in breakdown.items()}
    g_ms = sum(a.elapsed_time(b) for a, b, _, i8 in gev if i8) / reps
    g_flops = sum(f for _, _, f, i8 in gev if i8) / reps
    g_n = sum(1 for *_, i8 in gev if i8) // reps
    achieved = g_flops / (g_ms / 1e3) / 1e12 if g_ms > 0 else None
    peak = tf_burst
    lib = _lib.load()
    gm = (M, N, K) if wl == "gemm" else (2048, 2 * cfg.ffn // world, cfg.d)
    gemm_kernel = lib.npub_w8a16_kernel_name(*gm).decode()
    roof = {"kernel": gemm_kernel, "bound": "tensor", "achieved": achieved,
            "peak": peak, "unit": "TFLOP/s", "frac": (achieved / peak) if achieved else None,
            "peak_source": f"{peak_src} bf16 dense (burst)", "launches_per_step": g_n,
            "flops_per_launch": g_flops / g_n if g_n else None,
            "avg_launch_us": g_ms * 1e3 / g_n if g_n else None,
            "traffic": _traffic(wl), "share_of_step": (g_ms / ms_per_step) if ms_per_step else None}

    # e2e: same step through the public API with host buffers, copies inside the timed region
    h_ins = h_in if isinstance(h_in, list) else [h_in]
    d_outs = d_out if isinstance(d_out, list) else [d_out]
    h_hosts = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True).copy_(t) for t in h_ins]
    o_hosts = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in d_outs]
    e2e_ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    torch.cuda.synchronize()
    barrier()
    e2e_ev[0].record()
    for i in range(args.steps):
        if flush is not None:
            flush.fill_(1.0)
        for dst, src in zip(h_ins, h_hosts):
            dst.copy_(src, non_blocking=True)
        step()
        for dst, src in zip(o_hosts, d_outs):
            dst.copy_(src, non_blocking=True)
    e2e_ev[1].record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e2e_ev[0].elapsed_time(e2e_ev[1])
    t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item()) / args.steps
    e2e_val = units / (e2e_ms / 1e3) if not replicas else units * world / (e2e_ms / 1e3)
    h2d = sum(t.numel() * t.element_size() for t in h_ins)
    d2h = sum(t.numel() * t.element_size() for t in d_outs)

    out = None
    if rank == 0:
        out = {"metric": METRIC, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
               "scaling": "weak" if replicas else "strong", "vs_baseline": None,
               "dtype": "fp16 (fp32 math)" if wl == "vector" else "int8 x fp16 -> fp32 acc",
               "data": "synthetic (seeded; random-init weights)", "config": config,
               "roofline": roof,
               "e2e": {"value": e2e_val, "unit": unit, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
               "gpu_launches": int(launches), "clocks": clk.summary(),
               "launch": "cuda_graph" if graph is not None else "eager"}
        if wl == "layer":
            out["breakdown_us"] = breakdown
            flops = llama.layer_flops(cfg, 2048, 2048)
            out["layer_tflops"] = flops / (ms_per_step / 1e3) / 1e12
            out["layer_tensor_frac"] = out["layer_tflops"] * world / peak
        if wl == "vector":
            out["breakdown_us"] = breakdown
            iso = vector_isolated_us(dev, gen)
            per = {k: {"bytes": vb[k], "us": iso[k], "gbs": vb[k] / (iso[k] * 1e-6) / 1e9,
                       "frac": vb[k] / (iso[k] * 1e-6) / 1e9 / hbm} for k in vb}
            out["per_kernel"] = per
            out.pop("roofline_gemm", None)
            out["roofline"] = {"kernel": "softmax_kernel (causal rows, 16-byte vectors, block reductions)",
                               "bound": "hbm", "achieved": per["softmax"]["gbs"], "peak": hbm, "unit": "GB/s",
                               "frac": per["softmax"]["frac"], "peak_source": f"{peak_src} HBM copy bandwidth",
                               "bytes_per_launch": vb["softmax"], "avg_launch_us": breakdown["softmax"],
                               "traffic": _traffic("vector")}
        if wl == "decode":
            out["breakdown_us"] = breakdown
            by = llama.decode_bytes(cfg, B, ctx + 1)
            out["hbm_gbs"] = by / world / (ms_per_step / 1e3) / 1e9
            out["hbm_frac"] = out["hbm_gbs"] / hbm
            # the dominant kernel of a decode step is the KV-cache read (attention);
            # the W8A16 GEMM figures move to their own key
            kv = 2.0 * B * (cfg.kv_heads // world) * (ctx + 1) * cfg.head_dim * 2
            att_us = breakdown.get("attention") if breakdown else None
            a_gbs = kv / (att_us * 1e-6) / 1e9 if att_us else None
            out["roofline_gemm"] = roof
            out["roofline"] = {"kernel": "decode_attn_stream_kernel (bulk-copy K/V ring, per-warp online softmax)",
                               "bound": "hbm", "achieved": a_gbs, "peak": hbm, "unit": "GB/s",
                               "frac": a_gbs / hbm if a_gbs else None,
                               "peak_source": f"{peak_src} HBM copy bandwidth", "bytes_per_launch": kv,
                               "avg_launch_us": att_us,
                               "traffic": _traffic("decode") if (B, ctx) == (64, 4096) and world == 1 else None}
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        tp.close()
        dist.destroy_process_group()
    return out


def run_stack(args):
    """The 32-layer Llama-7B-shaped W8A16 stack: 32 prompts x 1024 tokens of
    prefill, then 128 greedy decode steps (one CUDA-graph replay each), tensor
    parallel over the ranks.  A step is prefill + decode; the metric counts
    prompt and generated tokens."""
    import torch
    sys.path.insert(0, HERE)
    from npu_comp_b200 import llama, npu, _lib
    rank, world, local = setup_dist(args.gpus)
    dev = torch.device("cuda", local)
    import torch.distributed as dist
    tp = llama.TP(rank, world, dist.group.WORLD if world > 1 else None)
    cfg = llama.LLAMA_7B
    B, T, S = 32, 1024, 128
    hbm, tf_burst, tf_sust, peak_src = _peaks()
    w = llama.make_stack(cfg, seed=0, device=dev, tp=tp)
    st = llama.LlamaStack(cfg, w, B, T, S, dev, tp)
    g = torch.Generator(device=dev)
    g.manual_seed(4321)
    prompts = torch.randint(0, cfg.vocab, (B, T), generator=g, device=dev, dtype=torch.int32)

    def barrier():
        if world > 1:
            dist.barrier()

    if args.ncu_region:
        st.prefill(prompts)
        st.decode(64)  # graph captured; KV length ~T + 64
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        if args.ncu_region == "prefill":
            st.prefill(prompts)
        else:
            st.decode(1)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print(json.dumps({"ncu_region": args.ncu_region, "workload": "llama7b_stack_w8a16"}))
        st.release()
        return
    for _ in range(args.warmup):
        st.prefill(prompts)
        st.decode(S)
    torch.cuda.synchronize()
    barrier()
    c0 = _lib.launch_count()
    st.prefill(prompts)
    prefill_launches = _lib.launch_count() - c0
    c0 = _lib.launch_count()
    st._decode_step()
    decode_launches = _lib.launch_count() - c0
    torch.cuda.synchronize()

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    try:
        smi_id = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        smi_id = local
    with ClockSampler(smi_id) as clk:
        clk.wait_first_sample()
        torch.cuda.synchronize()
        barrier()
        for i in range(args.steps):
            ev[i][0].record()
            st.prefill(prompts)
            ev[i][1].record()
            st.decode(S)
            ev[i][2].record()
        torch.cuda.synchronize()
        barrier()
    pre_ms = sum(e[0].elapsed_time(e[1]) for e in ev)
    dec_ms = sum(e[1].elapsed_time(e[2]) for e in ev)
    t = torch.tensor([pre_ms, dec_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    pre_ms, dec_ms = (float(v) / args.steps for v in t.tolist())
    ms_per_step = pre_ms + dec_ms
    tokens = B * (T + S)
    value = tokens / (ms_per_step / 1e3)

    # W8A16 GEMM roofline: the prefill's GEMM launches timed with CUDA events on their stream
    npu.gemm_events = []
    st.prefill(prompts)
    torch.cuda.synchronize()
    gev, npu.gemm_events = npu.gemm_events, None
    g_ms = sum(a.elapsed_time(b) for a, b, _, i8 in gev if i8)
    g_flops = sum(f for _, _, f, i8 in gev if i8)
    g_n = sum(1 for *_, i8 in gev if i8)
    achieved = g_flops / (g_ms / 1e3) / 1e12 if g_ms > 0 else None
    # the prefill GEMMs run back to back for hundreds of ms under the power cap:
    # the sustained figure is their denominator (burst is for a kernel timed alone)
    roof = {"kernel": "w8a16_pair_kernel (tcgen05 cta_group::2 W8A16)", "bound": "tensor", "achieved": achieved,
            "peak": tf_sust, "unit": "TFLOP/s", "frac": achieved / tf_sust if achieved else None,
            "peak_source": f"{peak_src} bf16 dense (sustained)", "launches_per_prefill": g_n,
            "avg_launch_us": g_ms * 1e3 / g_n if g_n else None, "traffic": _traffic("stack"),
            "share_of_prefill": g_ms / pre_ms if pre_ms else None}

    # e2e: prompts from pinned host memory in, generated tokens back to the host
    h_prompts = torch.empty((B, T), dtype=torch.int32, pin_memory=True)
    h_prompts.copy_(prompts)
    h_tokens = torch.empty((S + 1, B), dtype=torch.int32, pin_memory=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier()
    e0.record()
    for _ in range(args.steps):
        prompts.copy_(h_prompts, non_blocking=True)
        st.prefill(prompts)
        st.decode(S, record=True)
        h_tokens.copy_(torch.stack(st.tokens[-(S + 1):]), non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    t = torch.tensor([e0.elapsed_time(e1) / args.steps], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())

    out = None
    if rank == 0:
        flops = llama.stack_flops(cfg, B, T, S)
        kv_read = sum(2 * B * cfg.kv_heads * (T + s + 1) * cfg.head_dim * 2 for s in range(S)) * cfg.layers
        w_read = S * (cfg.layers * (cfg.d * (cfg.q_dim + 2 * cfg.kv_dim) + cfg.q_dim * cfg.d + 3 * cfg.d * cfg.ffn)
                      + 2 * cfg.vocab * cfg.d)
        out = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
               "vs_baseline": None, "dtype": "int8 x fp16 -> fp32 acc",
               "data": "synthetic (seeded prompts; random-init weights)",
               "config": {"workload": "llama7b_stack_w8a16", "layers": cfg.layers, "d": cfg.d, "heads": cfg.heads,
                          "head_dim": cfg.head_dim, "ffn": cfg.ffn, "vocab": cfg.vocab, "batch": B,
                          "prompt_len": T, "new_tokens": S, "parallelism": f"tp{world}",
                          "l2": "inputs larger than L2 (6.5 GB int8 weights, 19 GB KV cache per step)"},
               "prefill_ms": pre_ms, "decode_ms": dec_ms,
               "prefill_tokens_per_s": B * T / (pre_ms / 1e3), "decode_tokens_per_s": B * S / (dec_ms / 1e3),
               "stack_tflops": flops / (ms_per_step / 1e3) / 1e12,
               "decode_hbm_gbs": (kv_read + w_read) / world / (dec_ms / 1e3) / 1e9,
               "roofline": roof,
               "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": B * T * 4,
                       "d2h_bytes_per_step": (S + 1) * B * 4},
               "gpu_launches": int((prefill_launches + S * decode_launches) * args.steps),
               "clocks": clk.summary(), "launch": "decode steps replayed from a CUDA graph"
               if st.graph is not None else "eager"}
    st.release()
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        tp.close()
        dist.destroy_process_group()
    return out


def workload_config(args, world):
    """The `config` of a bench line: the same dict for both arms."""
    sys.path.insert(0, HERE)
    from npu_comp_b200.llama import LLAMA_7B as c
    wl = args.workload
    if wl == "stack":
        return {"workload": "llama7b_stack_w8a16", "layers": c.layers, "d": c.d, "heads": c.heads,
                "head_dim": c.head_dim, "ffn": c.ffn, "vocab": c.vocab, "batch": 32, "prompt_len": 1024,
                "new_tokens": 128, "parallelism": f"tp{world}",
                "l2": "inputs larger than L2 (6.5 GB int8 weights, 19 GB KV cache per step)"}
    if wl == "layer":
        return {"workload": "llama7b_layer_prefill_w8a16", "tokens": 2048, "batch": 1, "d": c.d, "heads": c.heads,
                "head_dim": c.head_dim, "ffn": c.ffn, "theta": c.theta, "parallelism": f"tp{world}",
                "l2": "inputs larger than L2 (202 MB int8 weights per step)"}
    if wl == "decode":
        return {"workload": "llama7b_layer_decode_w8a16", "batch": args.batch or 64, "kv_len": args.ctx or 4096,
                "parallelism": f"tp{world}", "l2": "inputs larger than L2 (4.3 GB KV cache per step)"}
    if wl == "vector":
        return {"workload": "llama_vector_ops_prefill", "rmsnorm": [2048, 4096], "swiglu": [2048, 11008],
                "softmax_causal": [32, 2048, 2048], "eps": 1e-5, "parallelism": f"replica{world}",
                "l2": "inputs larger than L2 (the softmax streams 403 MB between the other ops)"}
    M, N, K = (2048, 2 * c.ffn, c.d) if not args.shape else tuple(map(int, args.shape.split(",")))
    return {"workload": "w8a16_gemm", "M": M, "N": N, "K": K, "parallelism": f"replica{world}",
            "l2": "flushed: 256 MB buffer written between steps"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: 5 for the stack, else as many as ~0.6 s of device time)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["stack", "layer", "decode", "gemm", "vector"], default="stack")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--eager", action="store_true", help="launch every op from the host instead of a CUDA graph")
    ap.add_argument("--shape", default=None, help="gemm workload: M,N,K instead of the gate|up projection")
    ap.add_argument("--batch", type=int, default=None, help="decode workload: sequences (default 64)")
    ap.add_argument("--ctx", type=int, default=None, help="decode workload: KV length (default 4096)")
    ap.add_argument("--ncu-region", choices=["prefill", "decode"], default=None,
                    help="stack workload, 1 GPU: after warm-up, bracket one prefill or one graph-replayed decode "
                         "step (64 steps in) with cudaProfilerStart/Stop for ncu --profile-from-start off, "
                         "then exit without a bench line")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.steps is None and args.workload == "stack":
        args.steps = 5
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", args.gpus))

    if args.impl == "reference":
        # The reference's CPU path (mysim on the programs it emits) on all of
        # this host's cores; rank 0 only.  Each step is one bounded sample of
        # every op kind (~10-20 s); W untimed samples first (at most 3), then K
        # timed ones (at most 10), so the run stays within minutes.
        if rank != 0:
            return 0
        warm = min(args.warmup, 3)
        for _ in range(warm):
            mysim_rates(all_cores=True)
        samples = []
        for _ in range(max(1, min(args.steps or 5, 10))):
            rates, cores, kind, note = mysim_rates(all_cores=True)
            samples.append(reference_value(args.workload, rates)[0])
        value = statistics.median(samples)
        unit = reference_value(args.workload, rates)[1]
        sample = (f"mysim on the reference's programs, {cores} concurrent processes: {note}; the workload's time "
                  "projected from the measured rate of each op kind (matmul FLOPs, RMSNorm/SwiGLU/softmax/RoPE "
                  "elements)")
        line = {"impl": "reference", "metric": METRIC, "value": value, "unit": unit, "n_gpus": world,
                "steps": len(samples), "warmup": warm, "higher_is_better": True, "vs_baseline": None,
                "ms_per_step": None, "dtype": "fp16 NPU datapath (f32 accumulate)",
                "data": "synthetic (seeded)", "config": workload_config(args, world),
                "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": kind, "sample": sample},
                "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                "rates": {k: v for k, v in rates.items()}}
        if not args.no_cpu_baseline:
            line["cpu_baseline_torch"] = torch_cpu_baseline(args.workload, _shape(args))
        print(json.dumps(line), flush=True)
        return 0

    out = run_stack(args) if args.workload == "stack" else run_ours(args)
    if rank == 0 and out is not None:
        out["config"] = workload_config(args, world)
        if not args.no_cpu_baseline and world == 1:
            rates, cores, kind, note = mysim_rates(all_cores=False)
            v, u = reference_value(args.workload, rates)
            out["cpu_baseline"] = {"value": v, "unit": u, "cores": cores, "kind": kind,
                                   "sample": f"mysim, 1 process: {note}; projected from the per-op-kind rates"}
            out["cpu_baseline_torch"] = torch_cpu_baseline(args.workload, _shape(args))
        print(json.dumps(out), flush=True)
    return 0


def _shape(args):
    return tuple(map(int, args.shape.split(","))) if args.shape else None


if __name__ == "__main__":
    sys.exit(main())

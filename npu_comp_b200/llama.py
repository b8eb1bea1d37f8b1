"""Llama decoder layer and stack on libnpub kernels, W8A16 linears.

Structure of the reference layer (b_program_examples/llama_layer.py:1-7,
d_compiler/npu_compiler/model.py:64-112):

    h = x + Attn(RMSNorm(x))        GQA, RoPE (rotate_half), causal softmax
    y = h + FFN(RMSNorm(h))         SwiGLU: down(silu(x Wg) * (x Wu))

Linears follow the x @ W convention of the reference (W [K, N]); they are
stored quantised and K-major: Wq [N, K] int8 + scale [N] fp16.

Tensor parallelism (Megatron style, one process per GPU): QKV and gate/up are
column-parallel (each rank owns heads / FFN columns), O and down are
row-parallel (each rank owns the matching K slice) followed by one all-reduce
(sum) per block through torch.distributed (NCCL over NVLink).  The residual
adds run after the reductions: h = x + attn inside the second RMSNorm kernel,
y = h + ffn in a vector add.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

from . import npu


@dataclass(frozen=True)
class LlamaConfig:
    d: int = 4096
    heads: int = 32
    kv_heads: int = 32
    head_dim: int = 128
    ffn: int = 11008
    eps: float = 1e-5
    theta: float = 10000.0
    vocab: int = 32000
    layers: int = 32

    @property
    def q_dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    def linear_flops_per_token(self) -> int:
        """2 * (QKV + O + gate/up + down) MACs per token of one layer."""
        d = self.d
        return 2 * d * (self.q_dim + 2 * self.kv_dim) + 2 * self.q_dim * d + 2 * d * 2 * self.ffn + 2 * self.ffn * d


# Llama-7B shaped layer (the W8A16 prefill/decode/stack workloads).
LLAMA_7B = LlamaConfig()
# The reference's reduced layer (llama_layer.py:11-17): SEQ 8, D 64, 4 q heads,
# 2 kv heads, head_dim 16, FFN 128, eps 0.
REDUCED = LlamaConfig(d=64, heads=4, kv_heads=2, head_dim=16, ffn=128, eps=0.0, theta=10000.0, vocab=256, layers=1)


@dataclass
class LayerWeights:
    """One layer's weights as held by one tensor-parallel rank."""
    wqkv: torch.Tensor       # int8 [(hq + 2*hkv)*hd, d]   rows: q heads | k heads | v heads (local)
    sqkv: torch.Tensor       # fp16 [(hq + 2*hkv)*hd]
    wo: torch.Tensor         # int8 [d, hq*hd]   (local K slice)
    so: torch.Tensor         # fp16 [d]
    wgu: torch.Tensor        # int8 [2*f, d]     rows: gate (local) | up (local)
    sgu: torch.Tensor        # fp16 [2*f]
    wd: torch.Tensor         # int8 [d, f]       (local K slice)
    sd: torch.Tensor         # fp16 [d]
    g1: torch.Tensor         # fp16 [d]
    g2: torch.Tensor         # fp16 [d]
    heads: int               # local q heads
    kv_heads: int            # local kv heads
    ffn: int                 # local FFN width

    def weight_bytes(self) -> int:
        ts = (self.wqkv, self.sqkv, self.wo, self.so, self.wgu, self.sgu, self.wd, self.sd, self.g1, self.g2)
        return sum(t.numel() * t.element_size() for t in ts)


@dataclass
class TP:
    """Tensor-parallel context: rank/size and the process group (None = 1 GPU)."""
    rank: int = 0
    size: int = 1
    group: Optional[object] = None

    def all_reduce(self, t: torch.Tensor) -> None:
        if self.size > 1:
            import torch.distributed as dist
            dist.all_reduce(t, group=self.group)


def _shard_rows(q: torch.Tensor, s: torch.Tensor, blocks: List[range]) -> (torch.Tensor, torch.Tensor):
    idx = torch.cat([torch.arange(r.start, r.stop, device=q.device) for r in blocks])
    return q.index_select(0, idx).contiguous(), s.index_select(0, idx).contiguous()


def tp_ranges(cfg: LlamaConfig, rank: int, size: int) -> Dict[str, List[range]]:
    """This rank's slices of the layer's linears under tensor parallelism.

    qkv / gu: output-channel (row) ranges of the fused column-parallel weights
    [q heads | k heads | v heads] and [gate | up]; o / d: input (K) ranges of
    the row-parallel O and down projections."""
    if cfg.heads % size or cfg.kv_heads % size or cfg.ffn % size:
        raise ValueError(f"tp={size} must divide heads {cfg.heads}, kv_heads {cfg.kv_heads} and ffn {cfg.ffn}")
    hq, hk, f, hd = cfg.heads // size, cfg.kv_heads // size, cfg.ffn // size, cfg.head_dim
    qd, kd = cfg.q_dim, cfg.kv_dim
    r = rank
    return {
        "qkv": [range(r * hq * hd, (r + 1) * hq * hd), range(qd + r * hk * hd, qd + (r + 1) * hk * hd),
                range(qd + kd + r * hk * hd, qd + kd + (r + 1) * hk * hd)],
        "o": [range(r * hq * hd, (r + 1) * hq * hd)],
        "gu": [range(r * f, (r + 1) * f), range(cfg.ffn + r * f, cfg.ffn + (r + 1) * f)],
        "d": [range(r * f, (r + 1) * f)],
    }


def quantize_linear(W: torch.Tensor):
    """fp32 [K, N] -> (int8 [N, K], fp16 [N]) with the libnpub quantiser."""
    return npu.quantize_w8(W.contiguous())


def make_layer(cfg: LlamaConfig, seed: int, device, tp: TP = TP(), std: float = 0.02) -> LayerWeights:
    """Random-init layer (weights ~N(0, std), RMSNorm gains 1), quantised per
    output channel over the full matrix, then sliced to this rank's shard."""
    rg = tp_ranges(cfg, tp.rank, tp.size)
    hq, hk, f = cfg.heads // tp.size, cfg.kv_heads // tp.size, cfg.ffn // tp.size
    d = cfg.d
    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed))

    def rnd(k, m):
        return torch.randn((k, m), generator=gen, device=device, dtype=torch.float32) * std

    q, s = quantize_linear(rnd(d, cfg.q_dim + 2 * cfg.kv_dim))          # QKV, column parallel
    wqkv, sqkv = _shard_rows(q, s, rg["qkv"])
    q, so = quantize_linear(rnd(cfg.q_dim, d))                           # O, row parallel
    wo = q[:, rg["o"][0].start:rg["o"][0].stop].contiguous()
    q, s = quantize_linear(rnd(d, 2 * cfg.ffn))                          # gate | up, column parallel
    wgu, sgu = _shard_rows(q, s, rg["gu"])
    q, sd = quantize_linear(rnd(cfg.ffn, d))                             # down, row parallel
    wd = q[:, rg["d"][0].start:rg["d"][0].stop].contiguous()
    del q
    ones = torch.ones(d, dtype=torch.float16, device=device)
    return LayerWeights(wqkv, sqkv, wo, so, wgu, sgu, wd, sd, ones, ones.clone(), hq, hk, f)


def layer_from_float(cfg: LlamaConfig, W: Dict[str, torch.Tensor], device) -> LayerWeights:
    """Build a 1-rank layer from float weights in the reference's layout
    (model.py:44-61 / llama_layer.py:24-31): Wq{h} [d, hd], Wk{k}, Wv{k} [d, hd],
    Wo{h} [hd, d], Wg, Wu [d, f], Wd [f, d], Wn1, Wn2 [d]."""
    H, KV = cfg.heads, cfg.kv_heads
    f32 = lambda t: torch.as_tensor(t, dtype=torch.float32, device=device)  # noqa: E731
    Wqkv = torch.cat([f32(W[f"Wq{h}"]) for h in range(H)] + [f32(W[f"Wk{k}"]) for k in range(KV)]
                     + [f32(W[f"Wv{k}"]) for k in range(KV)], dim=1)
    wqkv, sqkv = quantize_linear(Wqkv)
    wo, so = quantize_linear(torch.cat([f32(W[f"Wo{h}"]) for h in range(H)], dim=0))
    wgu, sgu = quantize_linear(torch.cat([f32(W["Wg"]), f32(W["Wu"])], dim=1))
    wd, sd = quantize_linear(f32(W["Wd"]))
    g1 = f32(W["Wn1"]).reshape(-1).half()
    g2 = f32(W["Wn2"]).reshape(-1).half()
    return LayerWeights(wqkv, sqkv, wo, so, wgu, sgu, wd, sd, g1, g2, H, KV, cfg.ffn)


@dataclass
class Scratch:
    """Activation buffers reused across layers (allocated once per shape)."""
    bufs: Dict[str, torch.Tensor] = field(default_factory=dict)

    def get(self, name: str, shape, dtype=torch.float16, device="cuda") -> torch.Tensor:
        t = self.bufs.get(name)
        if t is None or tuple(t.shape) != tuple(shape) or t.dtype != dtype:
            t = torch.empty(shape, dtype=dtype, device=device)
            self.bufs[name] = t
        return t


class _Marks:
    """Optional per-op CUDA events: (name, start, end) appended to `events`."""

    def __init__(self, events):
        self.events = events
        self.cur = None

    def __call__(self, name):
        if self.events is None:
            return
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        if self.cur is not None:
            self.events.append((self.cur[0], self.cur[1], e))
        self.cur = (name, e)

    def end(self):
        self("")


def layer_prefill(x: torch.Tensor, w: LayerWeights, cfg: LlamaConfig, *, batch: int = 1, tp: TP = TP(),
                  positions: Optional[torch.Tensor] = None, kv_out: Optional[tuple] = None,
                  scratch: Optional[Scratch] = None, out: Optional[torch.Tensor] = None,
                  events: Optional[list] = None) -> torch.Tensor:
    """One decoder layer over `batch` prompts of equal length stacked in x [batch*T, d].

    kv_out: optional (k_cache, v_cache) [batch, kv_heads_local, cap, hd] that
    receive the prompt's (RoPE'd) K and V for later decode steps.
    """
    sc = scratch or Scratch()
    dev = x.device
    BT, d = x.shape
    T = BT // batch
    hd = cfg.head_dim
    hq, hk = w.heads, w.kv_heads
    qkv_n = (hq + 2 * hk) * hd
    if positions is None:
        positions = torch.arange(T, device=dev, dtype=torch.int32).repeat(batch)
    mk = _Marks(events)
    # attention block
    mk("rmsnorm")
    xn = npu.rmsnorm(x, w.g1, cfg.eps, out=sc.get("xn", (BT, d), device=dev))
    mk("qkv_gemm")
    qkv = npu.matmul(xn, w.wqkv, w.sqkv, out=sc.get("qkv", (BT, qkv_n), device=dev))
    q = qkv[:, : hq * hd]
    k = qkv[:, hq * hd:(hq + hk) * hd]
    v = qkv[:, (hq + hk) * hd:]
    mk("rope")
    npu.rope(qkv, hq + hk, hd, positions=positions, theta=cfg.theta)  # q and k heads are adjacent columns
    if kv_out is not None:
        _store_prompt_kv(k, v, kv_out, batch, T, hk, hd)
    mk("attention")
    ctx = npu.attention(q, k, v, hq, hk, head_dim=hd, batch=batch, causal=True,
                        out=sc.get("ctx", (BT, hq * hd), device=dev))
    mk("o_gemm")
    attn = npu.matmul(ctx, w.wo, w.so, out=sc.get("attn", (BT, d), device=dev))
    mk("all_reduce")
    tp.all_reduce(attn)
    # FFN block: h = x + attn is formed inside the RMSNorm kernel (llama_layer.py:139)
    mk("rmsnorm")
    h = sc.get("h", (BT, d), device=dev)
    hn, _ = npu.rmsnorm(attn, w.g2, cfg.eps, residual=x, residual_out=h, out=sc.get("hn", (BT, d), device=dev))
    mk("gate_up_gemm")
    gu = npu.matmul(hn, w.wgu, w.sgu, out=sc.get("gu", (BT, 2 * w.ffn), device=dev))
    mk("swiglu")
    a = npu.swiglu(gu, out=sc.get("act", (BT, w.ffn), device=dev))
    mk("down_gemm")
    ffn = npu.matmul(a, w.wd, w.sd, out=sc.get("ffn", (BT, d), device=dev))
    mk("all_reduce")
    tp.all_reduce(ffn)
    mk("residual")
    y = out if out is not None else torch.empty((BT, d), dtype=torch.float16, device=dev)
    npu.add(ffn, h, out=y)
    mk.end()
    return y


def _store_prompt_kv(k, v, kv_out, batch, T, hk, hd):
    kc, vc = kv_out
    # [batch*T, hk*hd] -> [batch, hk, T, hd] into the first T slots of the caches
    kc[:, :, :T, :].copy_(k.reshape(batch, T, hk, hd).transpose(1, 2))
    vc[:, :, :T, :].copy_(v.reshape(batch, T, hk, hd).transpose(1, 2))


def layer_decode(x: torch.Tensor, w: LayerWeights, cfg: LlamaConfig, k_cache: torch.Tensor, v_cache: torch.Tensor,
                 pos: torch.Tensor, *, ctx_max: int, tp: TP = TP(), scratch: Optional[Scratch] = None,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One decode step: x [B, d] holds one new token per sequence at positions
    pos [B] (int32); its K/V are appended to the caches, attention covers
    positions 0..pos[b]."""
    sc = scratch or Scratch()
    dev = x.device
    B, d = x.shape
    hd = cfg.head_dim
    hq, hk = w.heads, w.kv_heads
    xn = npu.rmsnorm(x, w.g1, cfg.eps, out=sc.get("dxn", (B, d), device=dev))
    qkv = npu.matmul(xn, w.wqkv, w.sqkv, out=sc.get("dqkv", (B, (hq + 2 * hk) * hd), device=dev))
    q = qkv[:, : hq * hd]
    k = qkv[:, hq * hd:(hq + hk) * hd]
    v = qkv[:, (hq + hk) * hd:]
    npu.rope(qkv, hq + hk, hd, positions=pos, theta=cfg.theta)  # q and k heads are adjacent columns
    npu.kv_append(k, v, k_cache, v_cache, pos=pos)
    lens = sc.get("dlens", (B,), dtype=torch.int32, device=dev)
    torch.add(pos, 1, out=lens)
    ctx = npu.attention_decode(q, k_cache, v_cache, heads=hq, kv_heads=hk, lens=lens, ctx_len=ctx_max,
                               out=sc.get("dctx", (B, hq * hd), device=dev))
    attn = npu.matmul(ctx, w.wo, w.so, out=sc.get("dattn", (B, d), device=dev))
    tp.all_reduce(attn)
    h = sc.get("dh", (B, d), device=dev)
    hn, _ = npu.rmsnorm(attn, w.g2, cfg.eps, residual=x, residual_out=h, out=sc.get("dhn", (B, d), device=dev))
    gu = npu.matmul(hn, w.wgu, w.sgu, out=sc.get("dgu", (B, 2 * w.ffn), device=dev))
    a = npu.swiglu(gu, out=sc.get("dact", (B, w.ffn), device=dev))
    ffn = npu.matmul(a, w.wd, w.sd, out=sc.get("dffn", (B, d), device=dev))
    tp.all_reduce(ffn)
    y = out if out is not None else torch.empty((B, d), dtype=torch.float16, device=dev)
    npu.add(ffn, h, out=y)
    return y


def layer_flops(cfg: LlamaConfig, tokens: int, ctx: int, causal: bool = True) -> float:
    """Algorithmic FLOPs of one layer over `tokens` query rows attending to `ctx` keys."""
    lin = cfg.linear_flops_per_token() * tokens
    pairs = tokens * ctx - (tokens * (tokens - 1) / 2 if causal else 0)
    attn = 4.0 * cfg.heads * cfg.head_dim * pairs
    return lin + attn


def decode_bytes(cfg: LlamaConfig, batch: int, ctx: int) -> float:
    """HBM bytes one decode step of one layer must move: int8 weights + scales,
    the KV cache read (ctx keys per sequence, K and V) and activations."""
    d, f = cfg.d, cfg.ffn
    w = d * (cfg.q_dim + 2 * cfg.kv_dim) + cfg.q_dim * d + d * 2 * f + f * d
    scales = 2 * ((cfg.q_dim + 2 * cfg.kv_dim) + d + 2 * f + d)
    kv = 2 * batch * cfg.kv_heads * ctx * cfg.head_dim * 2
    act = batch * 2 * (6 * d + (cfg.q_dim + 2 * cfg.kv_dim) * 2 + 3 * f * 2)
    return float(w + scales + kv + act)


def softmax_scale(cfg: LlamaConfig) -> float:
    return 1.0 / math.sqrt(cfg.head_dim)

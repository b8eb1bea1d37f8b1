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
import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

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
    # Llama-3 RoPE frequency scaling (legalize.py:50-64): (factor, low, high,
    # original context), or None for theta^(-2i/hd) alone
    rope_scaling: Optional[Tuple[float, float, float, float]] = None

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
# The reference's all-64-multiple layer (model.py:23-25): D 64, one head of 64, FFN 64.
MEDIUM = LlamaConfig(d=64, heads=1, kv_heads=1, head_dim=64, ffn=64, eps=1e-5, theta=10000.0, vocab=256, layers=1)
# The real Llama 3.2 3B layer of the reference (model.py:20-21): D 3072, 24 q /
# 8 kv heads of 128, FFN 8192, RoPE base 500000 with the Llama-3 scaling
# (legalize.py:50-64: factor 32, low 1, high 4, original context 8192); the
# 3B model's 28 layers and 128256-token vocabulary for the stack.
LLAMA_3_2_3B = LlamaConfig(d=3072, heads=24, kv_heads=8, head_dim=128, ffn=8192, eps=1e-5, theta=500000.0,
                           vocab=128256, layers=28, rope_scaling=(32.0, 1.0, 4.0, 8192.0))

_FREQS: Dict[tuple, torch.Tensor] = {}


def rope_inv_freq(cfg: LlamaConfig, device) -> Optional[torch.Tensor]:
    """The frequency table of a config with Llama-3 RoPE scaling (fp32 CUDA
    [head_dim/2], cached per device), None for plain theta frequencies.  Made
    on first use: call it (or run a prefill) before capturing a CUDA graph."""
    if cfg.rope_scaling is None:
        return None
    dev = torch.device(device)
    key = (cfg.head_dim, cfg.theta, tuple(cfg.rope_scaling), dev.type, dev.index)
    t = _FREQS.get(key)
    if t is None:
        t = npu.rope_freqs(cfg.head_dim, cfg.theta, llama3_scaling=tuple(cfg.rope_scaling), device=dev)
        _FREQS[key] = t
    return t


@dataclass
class LayerWeights:
    """One layer's weights as held by one tensor-parallel rank."""
    wqkv: torch.Tensor       # int8 [(hq + 2*hkv)*hd, d]   rows: q heads | k heads | v heads (local)
    sqkv: torch.Tensor       # fp16 [(hq + 2*hkv)*hd]
    wo: torch.Tensor         # int8 [d, hq*hd]   (local K slice)
    so: torch.Tensor         # fp16 [d]
    wgu: torch.Tensor        # int8 [2*f, d]     rows interleaved: 2c gate c, 2c+1 up c (local)
    sgu: torch.Tensor        # fp16 [2*f]        same order
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
    """Tensor-parallel context: rank/size and the process group (None = 1 GPU).

    all_reduce sums decode-sized fp16 tensors (<= 1 MB) with the NVLink
    peer-memory kernel of npu_comp_b200.comm and larger ones with NCCL."""
    rank: int = 0
    size: int = 1
    group: Optional[object] = None
    peer: Optional[object] = None

    def all_reduce(self, t: torch.Tensor) -> None:
        if self.size <= 1:
            return
        import torch.distributed as dist
        from . import comm
        if t.is_cuda:
            if self.peer is None and comm.enabled() and dist.get_backend(self.group) == "nccl":
                self.peer = comm.PeerAllReduce(self.group, t.device)
            if self.peer is not None and self.peer.fits(t):
                self.peer.all_reduce_(t)
                return
        dist.all_reduce(t, group=self.group)

    def close(self) -> None:
        if self.peer is not None:
            self.peer.close()
            self.peer = None


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


def _pack_layer(cfg: LlamaConfig, Wqkv: torch.Tensor, Wo: torch.Tensor, Wgu: torch.Tensor, Wd: torch.Tensor,
                g1: torch.Tensor, g2: torch.Tensor, tp: TP) -> LayerWeights:
    """Quantise the fused float linears (x @ W layout: Wqkv [d, (H+2KV)*hd],
    Wo [H*hd, d], Wgu [d, 2F] = [gate | up], Wd [F, d]) per output channel over
    the full matrices, then keep this rank's shard: output rows of the
    column-parallel QKV and gate|up (gate|up interleaved per rank), input
    columns (K) of the row-parallel O and down."""
    rg = tp_ranges(cfg, tp.rank, tp.size)
    hq, hk, f = cfg.heads // tp.size, cfg.kv_heads // tp.size, cfg.ffn // tp.size
    q, s = quantize_linear(Wqkv)                                         # QKV, column parallel
    wqkv, sqkv = _shard_rows(q, s, rg["qkv"])
    q, so = quantize_linear(Wo)                                          # O, row parallel
    wo = q[:, rg["o"][0].start:rg["o"][0].stop].contiguous()
    q, s = quantize_linear(Wgu)                                          # gate | up, column parallel
    wgu, sgu = npu.interleave_gate_up(*_shard_rows(q, s, rg["gu"]))
    q, sd = quantize_linear(Wd)                                          # down, row parallel
    wd = q[:, rg["d"][0].start:rg["d"][0].stop].contiguous()
    del q
    return LayerWeights(wqkv, sqkv, wo, so, wgu, sgu, wd, sd, g1.contiguous(), g2.contiguous(), hq, hk, f)


def make_layer(cfg: LlamaConfig, seed: int, device, tp: TP = TP(), std: float = 0.02) -> LayerWeights:
    """Random-init layer (weights ~N(0, std), RMSNorm gains 1), quantised per
    output channel over the full matrix, then sliced to this rank's shard."""
    d = cfg.d
    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed))

    def rnd(k, m):
        return torch.randn((k, m), generator=gen, device=device, dtype=torch.float32) * std

    # drawn in this order (QKV, O, gate|up, down) so a seed gives the same layer on every rank
    Wqkv = rnd(d, cfg.q_dim + 2 * cfg.kv_dim)
    Wo = rnd(cfg.q_dim, d)
    Wgu = rnd(d, 2 * cfg.ffn)
    Wd = rnd(cfg.ffn, d)
    ones = torch.ones(d, dtype=torch.float16, device=device)
    return _pack_layer(cfg, Wqkv, Wo, Wgu, Wd, ones, ones.clone(), tp)


def layer_from_float(cfg: LlamaConfig, W: Dict[str, torch.Tensor], device, tp: TP = TP()) -> LayerWeights:
    """Build this rank's layer from float weights in the reference's layout
    (model.py:44-61 / llama_layer.py:24-31): Wq{h} [d, hd], Wk{k}, Wv{k} [d, hd],
    Wo{h} [hd, d], Wg, Wu [d, f], Wd [f, d], Wn1, Wn2 [d].  The matrices are
    fused and quantised over their full size, then sharded for tp (heads, kv
    heads and FFN columns split evenly; GQA groups stay whole per rank)."""
    H, KV = cfg.heads, cfg.kv_heads
    f32 = lambda t: torch.as_tensor(t, dtype=torch.float32, device=device)  # noqa: E731
    Wqkv = torch.cat([f32(W[f"Wq{h}"]) for h in range(H)] + [f32(W[f"Wk{k}"]) for k in range(KV)]
                     + [f32(W[f"Wv{k}"]) for k in range(KV)], dim=1)
    Wo = torch.cat([f32(W[f"Wo{h}"]) for h in range(H)], dim=0)
    Wgu = torch.cat([f32(W["Wg"]), f32(W["Wu"])], dim=1)
    g1 = f32(W["Wn1"]).reshape(-1).half()
    g2 = f32(W["Wn2"]).reshape(-1).half()
    return _pack_layer(cfg, Wqkv, Wo, Wgu, f32(W["Wd"]), g1, g2, tp)


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
                  events: Optional[list] = None, residual: Optional[torch.Tensor] = None,
                  defer_residual: bool = False):
    """One decoder layer over `batch` prompts of equal length stacked in x [batch*T, d].

    kv_out: optional (k_cache, v_cache) [batch, kv_heads_local, cap, hd] that
    receive the prompt's (RoPE'd) K and V for later decode steps.
    residual / defer_residual: a stack of layers passes the previous layer's
    (ffn, h) pair unsummed -- the layer input is then fp16(x + residual), formed
    inside the first RMSNorm -- and defer_residual=True returns this layer's
    (ffn, h) instead of fp16(ffn + h); the same bits, one launch and one pass
    over the activations fewer per layer.
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
    if residual is None:
        xn = npu.rmsnorm(x, w.g1, cfg.eps, out=sc.get("xn", (BT, d), device=dev))
    else:
        xn, x = npu.rmsnorm(x, w.g1, cfg.eps, residual=residual, residual_out=sc.get("xres", (BT, d), device=dev),
                            out=sc.get("xn", (BT, d), device=dev))
    mk("qkv_gemm")
    qkv = npu.matmul(xn, w.wqkv, w.sqkv, out=sc.get("qkv", (BT, qkv_n), device=dev))
    q = qkv[:, : hq * hd]
    k = qkv[:, hq * hd:(hq + hk) * hd]
    v = qkv[:, (hq + hk) * hd:]
    mk("rope")
    if kv_out is not None:
        # q, k rotated in place and the prompt's K, V stored into the caches, one kernel
        npu.rope_kv_store(qkv, hq, hk, hd, positions, kv_out[0], kv_out[1], tokens_per_seq=T, theta=cfg.theta,
                          inv_freq=rope_inv_freq(cfg, dev))
    else:  # q and k heads are adjacent columns
        npu.rope(qkv, hq + hk, hd, positions=positions, theta=cfg.theta, inv_freq=rope_inv_freq(cfg, dev))
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
    mk("gate_up_gemm")  # SwiGLU in the GEMM epilogue (interleaved gate/up rows)
    a = npu.matmul_swiglu(hn, w.wgu, w.sgu, out=sc.get("act", (BT, w.ffn), device=dev))
    mk("down_gemm")
    ffn = npu.matmul(a, w.wd, w.sd, out=sc.get("ffn", (BT, d), device=dev))
    mk("all_reduce")
    tp.all_reduce(ffn)
    if defer_residual:
        mk.end()
        return ffn, h
    mk("residual")
    y = out if out is not None else torch.empty((BT, d), dtype=torch.float16, device=dev)
    npu.add(ffn, h, out=y)
    mk.end()
    return y


def llama_layer(x: torch.Tensor, weights, cfg: LlamaConfig, *, batch: int = 1, tp: TP = TP(),
                positions: Optional[torch.Tensor] = None, kv_out: Optional[tuple] = None,
                scratch: Optional[Scratch] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The Llama decoder layer under the reference's name (llama_layer.py:114-152:
    h = x + Attn(RMSNorm(x)); y = h + FFN(RMSNorm(h))) over `batch` prompts
    stacked in x [batch*T, d] fp16.

    weights: LayerWeights (make_layer / layer_from_float), or the reference's
    float weight dict (Wq{h}, Wk{k}, Wv{k}, Wo{h}, Wg, Wu, Wd, Wn1, Wn2 in the
    layout of llama_layer.py:24-31), which is quantised per output channel
    here and sharded for tp (every rank passes the full dict).  Same
    computation and bits as layer_prefill.
    """
    if not isinstance(weights, LayerWeights):
        weights = layer_from_float(cfg, weights, x.device, tp)
    elif tp.size > 1 and (weights.heads * tp.size != cfg.heads or weights.ffn * tp.size != cfg.ffn):
        raise ValueError(f"weights hold {weights.heads} of {cfg.heads} heads and {weights.ffn} of {cfg.ffn} FFN "
                         f"columns: not a shard for tp={tp.size}")
    return layer_prefill(x, weights, cfg, batch=batch, tp=tp, positions=positions, kv_out=kv_out, scratch=scratch,
                         out=out)


def layer_decode(x: torch.Tensor, w: LayerWeights, cfg: LlamaConfig, k_cache: torch.Tensor, v_cache: torch.Tensor,
                 pos: torch.Tensor, *, ctx_max: int, tp: TP = TP(), scratch: Optional[Scratch] = None,
                 out: Optional[torch.Tensor] = None, events: Optional[list] = None,
                 residual: Optional[torch.Tensor] = None, defer_residual: bool = False):
    """One decode step: x [B, d] holds one new token per sequence at positions
    pos [B] (int32); its K/V are appended to the caches, attention covers
    positions 0..pos[b].  residual / defer_residual as in layer_prefill."""
    sc = scratch or Scratch()
    dev = x.device
    B, d = x.shape
    hd = cfg.head_dim
    hq, hk = w.heads, w.kv_heads
    if residual is None and not defer_residual and folded_norm_ok(cfg, B, tp):
        mk = _Marks(events)
        mk("rmsnorm")
        g, ss = npu.rmsnorm_parts(x, w.g1, g_out=sc.get("dgA", (B, d), device=dev),
                                  ss_out=sc.get("dssA", (d // 32, B), torch.float32, dev))
        y, _, _ = layer_decode_folded(x, g, ss, w, cfg, k_cache, v_cache, pos, ctx_max=ctx_max, scratch=sc, out=out,
                                      mk=mk, tp=tp)
        mk.end()
        return y
    mk = _Marks(events)
    mk("rmsnorm")
    if residual is None:
        xn = npu.rmsnorm(x, w.g1, cfg.eps, out=sc.get("dxn", (B, d), device=dev))
    else:
        xn, x = npu.rmsnorm(x, w.g1, cfg.eps, residual=residual, residual_out=sc.get("dxres", (B, d), device=dev),
                            out=sc.get("dxn", (B, d), device=dev))
    mk("qkv_gemm")
    qkv = npu.matmul(xn, w.wqkv, w.sqkv, out=sc.get("dqkv", (B, (hq + 2 * hk) * hd), device=dev))
    q = qkv[:, : hq * hd]
    mk("rope_kv_append")
    lens = sc.get("dlens", (B,), dtype=torch.int32, device=dev)
    npu.rope_kv_append(qkv, hq, hk, hd, pos, k_cache, v_cache, theta=cfg.theta, lens=lens,
                       inv_freq=rope_inv_freq(cfg, dev))
    mk("attention")
    ctx = npu.attention_decode(q, k_cache, v_cache, heads=hq, kv_heads=hk, lens=lens, ctx_len=ctx_max,
                               out=sc.get("dctx", (B, hq * hd), device=dev))
    mk("o_gemm")
    attn = _row_parallel(ctx, w.wo, w.so, tp, sc.get("dattn", (B, d), device=dev), mk)
    mk("rmsnorm")
    h = sc.get("dh", (B, d), device=dev)
    hn, _ = npu.rmsnorm(attn, w.g2, cfg.eps, residual=x, residual_out=h, out=sc.get("dhn", (B, d), device=dev))
    mk("gate_up_gemm")  # SwiGLU in the GEMM epilogue (interleaved gate/up rows)
    a = npu.matmul_swiglu(hn, w.wgu, w.sgu, out=sc.get("dact", (B, w.ffn), device=dev))
    mk("down_gemm")
    ffn = _row_parallel(a, w.wd, w.sd, tp, sc.get("dffn", (B, d), device=dev), mk)
    if defer_residual:
        mk.end()
        return ffn, h
    mk("residual")
    y = out if out is not None else torch.empty((B, d), dtype=torch.float16, device=dev)
    npu.add(ffn, h, out=y)
    mk.end()
    return y


def folded_norm_ok(cfg: LlamaConfig, batch: int, tp: TP) -> bool:
    """Whether a decode step runs with its RMSNorms folded into the W8A16 GEMMs
    (npu.matmul_rms, the stream-K kernel): one rank (the row-parallel
    projections' all-reduce sits between a GEMM and the next norm otherwise),
    d a multiple of 32 and at most 32 sequences -- where the O and down
    projections run on the stream-K kernel anyway.  Measured on one B200
    (graph replay): a batch-32 Llama-7B decode layer step 222.7 -> 208.3 us,
    the stack's 128 decode steps 886.1 -> 835.8 ms; at batch 64, where the
    square and K-long projections run faster on the pair kernel, 752.8 ->
    765.7 us (so not there).  Under tensor parallelism the folding needs the
    peer all-reduce (npu_comp_b200.comm): it adds the residual and leaves the
    next RMSNorm's inputs itself.  NPUB_FOLD_RMSNORM=0 in the environment keeps
    the separate RMSNorm launches."""
    if os.environ.get("NPUB_FOLD_RMSNORM", "1") == "0" or batch > 32 or cfg.d % 32:
        return False
    if tp.size == 1:
        return True
    return tp.peer is not None and batch * cfg.d * 2 <= tp.peer.max_bytes


def layer_decode_folded(h: torch.Tensor, g: torch.Tensor, ss: torch.Tensor, w: LayerWeights, cfg: LlamaConfig,
                        k_cache: torch.Tensor, v_cache: torch.Tensor, pos: torch.Tensor, *, ctx_max: int,
                        scratch: Scratch, gamma_next: Optional[torch.Tensor] = None,
                        out: Optional[torch.Tensor] = None, out_g: Optional[torch.Tensor] = None,
                        out_ss: Optional[torch.Tensor] = None, mk=None, tp: TP = TP(),
                        w_next: Optional[LayerWeights] = None):
    """One decode step of a layer (llama_layer.py:71-152) with both RMSNorms
    folded into the GEMMs: h is the residual stream entering the layer and
    (g, ss) = rmsnorm_parts(h, w.g1) or the previous layer's down projection's
    outputs.  The O projection adds h and leaves (h2, g2, ss2) for the gate|up
    projection; the down projection adds h2 and, with gamma_next (the next
    RMSNorm's weight), leaves (g, ss) for the next layer.  Returns (y, g', ss').
    Under tensor parallelism the row-parallel O and down projections store
    their partial sums and the peer all-reduce adds the residual and makes
    the next RMSNorm's inputs.  Each GEMM prefetches the first weight tiles of
    the next one to L2 (w_next: the next layer, for its QKV projection);
    NPUB_PREFETCH_NEXT=0 in the environment turns that off."""
    sc = scratch
    pf = os.environ.get("NPUB_PREFETCH_NEXT", "1") != "0"
    mk = mk or _Marks(None)
    dev = h.device
    B, d = h.shape
    hd = cfg.head_dim
    hq, hk = w.heads, w.kv_heads
    mk("qkv_gemm")
    qkv = npu.matmul_rms(g, w.wqkv, w.sqkv, rs=(ss, d), eps=cfg.eps,
                         out=sc.get("dqkv", (B, (hq + 2 * hk) * hd), device=dev))
    q = qkv[:, : hq * hd]
    mk("rope_kv_append")
    lens = sc.get("dlens", (B,), dtype=torch.int32, device=dev)
    npu.rope_kv_append(qkv, hq, hk, hd, pos, k_cache, v_cache, theta=cfg.theta, lens=lens,
                       inv_freq=rope_inv_freq(cfg, dev))
    mk("attention")
    ctx = npu.attention_decode(q, k_cache, v_cache, heads=hq, kv_heads=hk, lens=lens, ctx_len=ctx_max,
                               out=sc.get("dctx", (B, hq * hd), device=dev))
    mk("o_gemm")
    h2, g2, ss2 = sc.get("dh", (B, d), device=dev), sc.get("dg2", (B, d), device=dev), \
        sc.get("dss2", (d // 32, B), torch.float32, dev)
    if tp.size > 1:
        part = npu.matmul(ctx, w.wo, w.so, out=sc.get("dattn", (B, d), device=dev))
        mk("all_reduce")
        tp.peer.all_reduce_rms(part, h, w.g2, h2, g2, ss2)
    else:
        npu.matmul_rms(ctx, w.wo, w.so, residual=h, gamma=w.g2, out=h2, g_out=g2, ss_out=ss2,
                       prefetch_next=w.wgu if pf else None)
    mk("gate_up_gemm")
    a = npu.matmul_rms(g2, w.wgu, w.sgu, swiglu=True, rs=(ss2, d), eps=cfg.eps,
                       out=sc.get("dact", (B, w.ffn), device=dev), prefetch_next=w.wd if pf else None)
    mk("down_gemm")
    y = out if out is not None else torch.empty((B, d), dtype=torch.float16, device=dev)
    if tp.size > 1:
        part = npu.matmul(a, w.wd, w.sd, out=sc.get("dffn", (B, d), device=dev))
        mk("all_reduce")
        gn = out_g if out_g is not None else sc.get("dgn", (B, d), device=dev)
        ssn = out_ss if out_ss is not None else sc.get("dssn", (d // 32, B), torch.float32, dev)
        # without a next norm (the last layer) the inputs are made and not used
        tp.peer.all_reduce_rms(part, h2, gamma_next if gamma_next is not None else w.g1, y, gn, ssn)
        return (y, gn, ssn) if gamma_next is not None else (y, None, None)
    nxt = w_next.wqkv if (pf and w_next is not None) else None
    if gamma_next is None:
        npu.matmul_rms(a, w.wd, w.sd, residual=h2, out=y, prefetch_next=nxt)
        return y, None, None
    _, gn, ssn = npu.matmul_rms(a, w.wd, w.sd, residual=h2, gamma=gamma_next, out=y, g_out=out_g, ss_out=out_ss,
                                prefetch_next=nxt)
    return y, gn, ssn


def _row_parallel(a: torch.Tensor, wq: torch.Tensor, s: torch.Tensor, tp: TP, out: torch.Tensor, mk) -> torch.Tensor:
    """Row-parallel projection of a decode step followed by its all-reduce."""
    npu.matmul(a, wq, s, out=out)
    mk("all_reduce")
    tp.all_reduce(out)
    return out


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


# ---------------------------------------------------------------------------
# The full decoder stack: embedding -> L layers -> final RMSNorm -> lm_head ->
# greedy argmax.  Prefill runs all prompts of a batch at once and fills the
# per-layer KV caches; decode appends one token per sequence per step.


@dataclass
class StackWeights:
    layers: List[LayerWeights]
    embed: torch.Tensor      # fp16 [vocab, d], replicated on every rank
    norm: torch.Tensor       # fp16 [d]
    lm_head: torch.Tensor    # fp16 [vocab / tp, d]: this rank's vocabulary rows (K-major for the GEMM)
    vocab_off: int


def make_stack(cfg: LlamaConfig, seed: int, device, tp: TP = TP(), layers: Optional[int] = None) -> StackWeights:
    """Random-init Llama-shaped stack: W8A16 layers (make_layer), an fp16 embedding
    table ~N(0, 1) and an fp16 lm_head ~N(0, 0.02) split over the vocabulary."""
    n_layers = cfg.layers if layers is None else layers
    if cfg.vocab % tp.size:
        raise ValueError(f"tp={tp.size} must divide the vocabulary {cfg.vocab}")
    lw = [make_layer(cfg, seed + 1000 * (i + 1), device, tp) for i in range(n_layers)]
    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed) + 7)
    embed = torch.randn((cfg.vocab, cfg.d), generator=gen, device=device).half()
    lm = torch.randn((cfg.vocab, cfg.d), generator=gen, device=device) * 0.02
    vs = cfg.vocab // tp.size
    lm_shard = lm[tp.rank * vs:(tp.rank + 1) * vs].half().contiguous()
    del lm
    return StackWeights(lw, embed, torch.ones(cfg.d, dtype=torch.float16, device=device), lm_shard, tp.rank * vs)


class LlamaStack:
    """A batch of `batch` sequences through the stack on this rank.

    prefill(prompts [B, T] int32) fills the KV caches and returns the first
    generated token of every sequence; decode(steps) generates `steps` more,
    replaying one CUDA graph per step (token ids and positions stay on the
    device, so the host only launches the graph)."""

    def __init__(self, cfg: LlamaConfig, w: StackWeights, batch: int, prompt_len: int, max_new: int, device,
                 tp: TP = TP(), use_graph: bool = True):
        self.cfg, self.w, self.tp, self.dev = cfg, w, tp, device
        self.B, self.T = batch, prompt_len
        self.cap = prompt_len + max_new + 1
        hk = cfg.kv_heads // tp.size
        kv_shape = (batch, hk, self.cap, cfg.head_dim)
        self.kc = [torch.zeros(kv_shape, dtype=torch.float16, device=device) for _ in w.layers]
        self.vc = [torch.zeros(kv_shape, dtype=torch.float16, device=device) for _ in w.layers]
        self.sc = Scratch()
        self.ids = torch.zeros((batch,), dtype=torch.int32, device=device)
        self.pos = torch.zeros((batch,), dtype=torch.int32, device=device)
        self.tokens: List[torch.Tensor] = []
        self.use_graph = use_graph
        self.graph = None
        self.positions = torch.arange(prompt_len, device=device, dtype=torch.int32).repeat(batch)
        rope_inv_freq(cfg, device)  # made here, outside any graph capture
        if tp.size > 1 and tp.peer is None:  # set up outside any graph capture
            import torch.distributed as dist
            from . import comm
            if comm.enabled() and dist.get_backend(tp.group) == "nccl":
                tp.peer = comm.PeerAllReduce(tp.group, device)

    # -- greedy selection over the (possibly vocab-sharded) lm_head
    def _next_ids(self, xl: torch.Tensor, residual: Optional[torch.Tensor] = None) -> None:
        cfg, w, tp, sc = self.cfg, self.w, self.tp, self.sc
        B = xl.shape[0]
        if residual is None:
            hn = npu.rmsnorm(xl, w.norm, cfg.eps, out=sc.get("fn", (B, cfg.d), device=self.dev))
        else:  # the last layer's residual add, inside the final RMSNorm
            hn, _ = npu.rmsnorm(xl, w.norm, cfg.eps, residual=residual,
                                residual_out=sc.get("fres", (B, cfg.d), device=self.dev),
                                out=sc.get("fn", (B, cfg.d), device=self.dev))
        logits = npu.matmul(hn, w.lm_head, out=sc.get("logits", (B, w.lm_head.shape[0]), device=self.dev))
        if tp.size == 1:
            npu.argmax(logits, idx=self.ids, val=sc.get("amax_v", (B,), torch.float32, self.dev))
            return
        # one (value, global index) key per row and shard, one all-gather, one
        # selection kernel: the largest value, the smallest index on ties
        import torch.distributed as dist
        keys = npu.argmax_keys(logits, w.vocab_off, keys=sc.get("amax_k", (B,), torch.int64, self.dev))
        all_k = sc.get("all_k", (tp.size * B,), torch.int64, self.dev)
        dist.all_gather_into_tensor(all_k, keys, group=tp.group)
        npu.select_keys(all_k, tp.size, ids=self.ids)

    def prefill(self, prompts: torch.Tensor) -> torch.Tensor:
        cfg, B, T = self.cfg, self.B, self.T
        x = npu.embed(prompts.reshape(-1), self.w.embed, out=self.sc.get("px0", (B * T, cfg.d), device=self.dev))
        res = None
        for i, lw in enumerate(self.w.layers):
            # each layer's residual add is folded into the next layer's first RMSNorm
            x, res = layer_prefill(x, lw, cfg, batch=B, tp=self.tp, positions=self.positions,
                                   kv_out=(self.kc[i], self.vc[i]), scratch=self.sc, residual=res,
                                   defer_residual=True)
        # the last layer's residual add, for the last prompt rows only
        xl = self.sc.get("xlast", (B, cfg.d), device=self.dev)
        npu.add(x.view(B, T, cfg.d)[:, T - 1], res.view(B, T, cfg.d)[:, T - 1], out=xl)
        self._next_ids(xl)
        self.pos.fill_(T)
        self.tokens = [self.ids.clone()]
        return self.ids

    def _decode_step(self) -> None:
        cfg, B = self.cfg, self.B
        x = npu.embed(self.ids, self.w.embed, out=self.sc.get("dx0", (B, cfg.d), device=self.dev))
        if folded_norm_ok(cfg, B, self.tp):
            # RMSNorms folded into the GEMMs: (h, g, ss) flow from layer to layer,
            # ping-ponging between two sets of buffers
            sc, d, dev, L = self.sc, cfg.d, self.dev, len(self.w.layers)
            g, ss = npu.rmsnorm_parts(x, self.w.layers[0].g1, g_out=sc.get("sg0", (B, d), device=dev),
                                      ss_out=sc.get("sss0", (d // 32, B), torch.float32, dev))
            h = x
            for i, lw in enumerate(self.w.layers):
                j = (i + 1) % 2
                nxt = self.w.layers[i + 1].g1 if i + 1 < L else None
                h, g, ss = layer_decode_folded(
                    h, g, ss, lw, cfg, self.kc[i], self.vc[i], self.pos, ctx_max=self.cap, scratch=sc,
                    gamma_next=nxt, out=sc.get(f"sh{j}", (B, d), device=dev),
                    out_g=sc.get(f"sg{j}", (B, d), device=dev),
                    out_ss=sc.get(f"sss{j}", (d // 32, B), torch.float32, dev), tp=self.tp,
                    w_next=self.w.layers[i + 1] if i + 1 < L else None)
            self._next_ids(h)
            self.pos.add_(1)
            return
        res = None
        for i, lw in enumerate(self.w.layers):
            x, res = layer_decode(x, lw, cfg, self.kc[i], self.vc[i], self.pos, ctx_max=self.cap, tp=self.tp,
                                  scratch=self.sc, residual=res, defer_residual=True)
        self._next_ids(x, res)
        self.pos.add_(1)

    def _capture(self) -> None:
        ids0, pos0 = self.ids.clone(), self.pos.clone()
        side = torch.cuda.Stream(device=self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(side):  # warm-up outside capture (allocations, first-launch set-up)
            self._decode_step()
        torch.cuda.current_stream(self.dev).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._decode_step()
        self.ids.copy_(ids0)
        self.pos.copy_(pos0)
        self.graph = g

    def decode(self, steps: int, record: bool = False) -> None:
        if self.use_graph and self.graph is None:
            try:
                self._capture()
            except Exception:
                self.graph = None
                self.use_graph = False
        for _ in range(steps):
            if self.graph is not None:
                self.graph.replay()
            else:
                self._decode_step()
            if record:
                self.tokens.append(self.ids.clone())

    def release(self) -> None:
        """Drop the CUDA graph (it may hold collectives) before the process group ends."""
        self.graph = None


def stack_flops(cfg: LlamaConfig, batch: int, prompt_len: int, new_tokens: int, layers: Optional[int] = None) -> float:
    """Algorithmic FLOPs of prefill + greedy decode of the stack (layers and lm_head)."""
    L = cfg.layers if layers is None else layers
    pre = L * batch * layer_flops(cfg, prompt_len, prompt_len) + 2.0 * batch * cfg.d * cfg.vocab
    dec = 0.0
    for s in range(new_tokens):
        ctx = prompt_len + s + 1
        dec += L * batch * layer_flops(cfg, 1, ctx, causal=False) + 2.0 * batch * cfg.d * cfg.vocab
    return pre + dec

"""The Llama layer (W8A16 linears, RoPE, causal GQA attention, SwiGLU) on the
GPU against the oracle.  Tolerance: normwise relative error <= 1e-2 (TOL)."""
import numpy as np
import pytest
import torch

import npu_comp_b200 as nb
from npu_comp_b200 import llama
from oracle import ref

pytestmark = pytest.mark.gpu
TOL = 1e-2


def layer_weights_from_fixture(ex):
    SEQ, D, H, KV, HD, F = (int(v) for v in ex["layer_dims"])
    W = {"Wn1": ex["layer_Wn1"], "Wn2": ex["layer_Wn2"], "Wg": ex["layer_Wg"], "Wu": ex["layer_Wu"],
         "Wd": ex["layer_Wd"]}
    for h in range(H):
        W[f"Wq{h}"] = ex["layer_Wq"][h]
        W[f"Wo{h}"] = ex["layer_Wo"][h]
    for k in range(KV):
        W[f"Wk{k}"] = ex["layer_Wk"][k]
        W[f"Wv{k}"] = ex["layer_Wv"][k]
    return W, (SEQ, D, H, KV, HD, F)


def test_reference_llama_layer(cuda_device, examples):
    """The reference's full layer (llama_layer.py: SEQ 8, D 64, H 4, KV 2, HD 16,
    F 128, eps 0) with its own weights, W8A16-quantised, vs its float reference
    and vs its NPU (mysim) result."""
    W, (SEQ, D, H, KV, HD, F) = layer_weights_from_fixture(examples)
    cfg = llama.LlamaConfig(d=D, heads=H, kv_heads=KV, head_dim=HD, ffn=F, eps=0.0, theta=10000.0, vocab=64,
                            layers=1)
    w = llama.layer_from_float(cfg, W, cuda_device)
    x = torch.from_numpy(examples["layer_X"]).half().to(cuda_device)
    y = llama.layer_prefill(x, w, cfg).float().cpu().numpy()
    assert ref.rel_err(y, examples["layer_ref"]) <= TOL           # llama_layer.py:199-205 uses 5e-2
    assert ref.rel_err(y, examples["layer_npu"]) <= TOL
    cos, sin = ref.rope_tables(SEQ, HD)
    yq = ref.ref_layer(ref.quantized_weights(W, H, KV), examples["layer_X"], H, KV, HD, 0.0, cos, sin)
    assert ref.rel_err(y, yq) <= 5e-3                                # same weights the GPU applies


def test_llama_layer_entry_point(cuda_device, examples):
    """npu_comp_b200.llama_layer, the reference's name for the layer, takes the
    reference's float weight dict directly and gives layer_prefill's bits."""
    W, (SEQ, D, H, KV, HD, F) = layer_weights_from_fixture(examples)
    cfg = llama.LlamaConfig(d=D, heads=H, kv_heads=KV, head_dim=HD, ffn=F, eps=0.0, theta=10000.0, vocab=64,
                            layers=1)
    x = torch.from_numpy(examples["layer_X"]).half().to(cuda_device)
    y = nb.llama_layer(x, W, cfg)
    w = llama.layer_from_float(cfg, W, cuda_device)
    assert torch.equal(y, llama.layer_prefill(x, w, cfg))
    assert torch.equal(y, nb.llama_layer(x, w, cfg))
    assert ref.rel_err(y.float().cpu().numpy(), examples["layer_ref"]) <= TOL


def random_float_layer(cfg, rng, std=0.02):
    W = {"Wn1": 1 + 0.02 * rng.standard_normal(cfg.d), "Wn2": 1 + 0.02 * rng.standard_normal(cfg.d),
         "Wg": rng.standard_normal((cfg.d, cfg.ffn)) * std, "Wu": rng.standard_normal((cfg.d, cfg.ffn)) * std,
         "Wd": rng.standard_normal((cfg.ffn, cfg.d)) * std}
    for h in range(cfg.heads):
        W[f"Wq{h}"] = rng.standard_normal((cfg.d, cfg.head_dim)) * std
        W[f"Wo{h}"] = rng.standard_normal((cfg.head_dim, cfg.d)) * std
    for k in range(cfg.kv_heads):
        W[f"Wk{k}"] = rng.standard_normal((cfg.d, cfg.head_dim)) * std
        W[f"Wv{k}"] = rng.standard_normal((cfg.d, cfg.head_dim)) * std
    return {k: v.astype(np.float32) for k, v in W.items()}


def test_llama7b_shaped_layer(cuda_device):
    """Llama-7B layer shape (d 4096, 32 x 128 heads, FFN 11008) at 128 tokens vs
    the float64 layer reference on the dequantised weights."""
    rng = np.random.default_rng(21)
    cfg = llama.LLAMA_7B
    W = random_float_layer(cfg, rng)
    x = rng.standard_normal((128, cfg.d)).astype(np.float16)
    w = llama.layer_from_float(cfg, W, cuda_device)
    y = llama.layer_prefill(torch.from_numpy(x).to(cuda_device), w, cfg).float().cpu().numpy()
    cos, sin = ref.rope_tables(128, cfg.head_dim)
    yr = ref.ref_layer(ref.quantized_weights(W, cfg.heads, cfg.kv_heads), x, cfg.heads, cfg.kv_heads,
                       cfg.head_dim, cfg.eps, cos, sin)
    assert ref.rel_err(y, yr) <= TOL
    assert np.abs(y - yr).mean() < 5e-3


def test_full_size_layer_properties(cuda_device):
    """T = 2048 prefill: deterministic, finite, and causal (changing the last
    tokens leaves earlier rows bit-identical)."""
    cfg = llama.LLAMA_7B
    w = llama.make_layer(cfg, seed=0, device=cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(1)
    x = torch.randn((2048, cfg.d), generator=g, device=cuda_device).half()
    y1 = llama.layer_prefill(x, w, cfg)
    y2 = llama.layer_prefill(x, w, cfg)
    assert torch.equal(y1, y2)
    assert torch.isfinite(y1).all()
    x2 = x.clone()
    x2[1900:] = torch.randn((148, cfg.d), generator=g, device=cuda_device).half()
    y3 = llama.layer_prefill(x2, w, cfg)
    assert torch.equal(y1[:1900], y3[:1900])  # causal: rows before the changed tokens are untouched
    assert not torch.equal(y1[1900:], y3[1900:])


def test_batched_prefill_equals_single_prompts(cuda_device):
    cfg = llama.LlamaConfig(d=256, heads=4, kv_heads=2, head_dim=64, ffn=512, eps=1e-5, theta=10000.0, vocab=64,
                            layers=1)
    w = llama.make_layer(cfg, seed=3, device=cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(2)
    x = torch.randn((3 * 40, cfg.d), generator=g, device=cuda_device).half()
    yb = llama.layer_prefill(x, w, cfg, batch=3).float()
    for b in range(3):
        ys = llama.layer_prefill(x[b * 40:(b + 1) * 40].contiguous(), w, cfg).float()
        e = ((yb[b * 40:(b + 1) * 40] - ys).abs().max() / ys.abs().max()).item()
        assert e <= 2e-3


def test_decode_step_matches_reference_and_prefill(cuda_device):
    """Llama-7B layer: prefill of T = 127 tokens per sequence fills the KV cache,
    then one decode step for token T.  The decode row must match row T of the
    float64 layer reference over T + 1 tokens (TOL), and row T of a GPU prefill
    over T + 1 tokens (two fp16 paths, each within TOL of the reference: 2 TOL)."""
    rng = np.random.default_rng(5)
    cfg = llama.LLAMA_7B
    W = random_float_layer(cfg, rng)
    w = llama.layer_from_float(cfg, W, cuda_device)
    B, T = 2, 127
    x = rng.standard_normal((B, T + 1, cfg.d)).astype(np.float16)
    xt = torch.from_numpy(x).to(cuda_device)
    full = llama.layer_prefill(xt.reshape(B * (T + 1), cfg.d), w, cfg, batch=B).float().view(B, T + 1, cfg.d)
    kc = torch.zeros((B, cfg.kv_heads, 256, cfg.head_dim), dtype=torch.float16, device=cuda_device)
    vc = torch.zeros_like(kc)
    llama.layer_prefill(xt[:, :T].reshape(B * T, cfg.d).contiguous(), w, cfg, batch=B, kv_out=(kc, vc))
    pos = torch.full((B,), T, dtype=torch.int32, device=cuda_device)
    yd = llama.layer_decode(xt[:, T].contiguous(), w, cfg, kc, vc, pos, ctx_max=T + 1).float()
    cos, sin = ref.rope_tables(T + 1, cfg.head_dim)
    qw = ref.quantized_weights(W, cfg.heads, cfg.kv_heads)
    for b in range(B):
        yr = ref.ref_layer(qw, x[b], cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.eps, cos, sin)[T]
        assert ref.rel_err(yd[b].cpu().numpy(), yr) <= TOL
    e = ((yd - full[:, T]).abs().max() / full[:, T].abs().max()).item()
    assert e <= 2 * TOL


def test_decode_folded_norms_match_separate_norms(cuda_device, monkeypatch):
    """A decode step with the RMSNorms folded into the GEMMs (npu.matmul_rms)
    and the same step with separate RMSNorm launches (NPUB_FOLD_RMSNORM=0):
    two fp16 paths of the same layer, batch 32 (the stack's decode batch)."""
    cfg = llama.LLAMA_7B
    w = llama.make_layer(cfg, seed=2, device=cuda_device)
    B, ctx = 32, 300
    g = torch.Generator(device=cuda_device).manual_seed(4)
    kc = torch.randn((B, cfg.kv_heads, ctx + 8, cfg.head_dim), generator=g, device=cuda_device).half()
    vc = torch.randn_like(kc)
    x = torch.randn((B, cfg.d), generator=g, device=cuda_device).half()
    pos = torch.full((B,), ctx, dtype=torch.int32, device=cuda_device)
    assert llama.folded_norm_ok(cfg, B, llama.TP())
    y1 = llama.layer_decode(x, w, cfg, kc.clone(), vc.clone(), pos, ctx_max=ctx + 1).float()
    monkeypatch.setenv("NPUB_FOLD_RMSNORM", "0")
    assert not llama.folded_norm_ok(cfg, B, llama.TP())
    y0 = llama.layer_decode(x, w, cfg, kc.clone(), vc.clone(), pos, ctx_max=ctx + 1).float()
    e = ((y1 - y0).abs().max() / y0.abs().max()).item()
    assert e <= TOL, e

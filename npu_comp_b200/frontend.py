"""PyTorch import frontend: trained Llama modules -> W8A16 weights for this
library (the role of d_compiler/npu_compiler/frontend.py:15-23, which hands a
torch nn.Module to TVM; here the module's parameters are quantised and packed
directly, since there is no program to compile).

Accepted inputs are plain `torch.nn.Linear` layers and Llama decoder layers /
models with the usual parameter names (a Hugging Face LlamaDecoderLayer or
LlamaForCausalLM, or their state_dicts):

    self_attn.{q,k,v,o}_proj.weight, mlp.{gate,up,down}_proj.weight,
    input_layernorm.weight, post_attention_layernorm.weight
    model.embed_tokens.weight, model.layers.<i>.*, model.norm.weight, lm_head.weight

nn.Linear keeps its weight as [out, in] and computes x @ weight.T, so the
reference's x @ W matrix (llama_layer.py:24-31) is weight.T and the
quantiser's K-major output [N, K] has the layout of weight itself.  The q/k
projections are taken as they are stored: the Hugging Face checkpoints
already use the rotate_half RoPE convention of the reference
(llama_layer.py:33-40), which is what the kernels implement.
"""
from __future__ import annotations

from typing import Dict, Mapping, Optional

import torch

from . import npu
from .llama import TP, LayerWeights, LlamaConfig, StackWeights, _pack_layer

_LAYER_KEYS = ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
               "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight",
               "input_layernorm.weight", "post_attention_layernorm.weight")


def quantize_linear(linear: torch.nn.Linear, device=None):
    """nn.Linear (no bias) -> (int8 [out, in], fp16 scale [out]): the W8A16
    per-output-channel quantisation of its weight, ready for npu.matmul
    (y = x @ weight.T becomes npu.matmul(x, q, s))."""
    if not isinstance(linear, torch.nn.Linear):
        raise TypeError(f"expected torch.nn.Linear, got {type(linear).__name__}")
    if linear.bias is not None:
        raise ValueError("a Linear with a bias is not a W8A16 matmul (the NPU op has no bias term)")
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    W = linear.weight.detach().to(device=dev, dtype=torch.float32).t().contiguous()  # x @ W layout [in, out]
    return npu.quantize_w8(W)


def config_from_hf(hf) -> LlamaConfig:
    """LlamaConfig from a Hugging Face LlamaConfig (or any object with its
    attribute names): sizes, eps, RoPE base and the llama3 frequency scaling."""
    heads = int(hf.num_attention_heads)
    d = int(hf.hidden_size)
    hd = int(getattr(hf, "head_dim", None) or d // heads)
    rp = getattr(hf, "rope_parameters", None) or getattr(hf, "rope_scaling", None) or {}
    theta = float(rp.get("rope_theta", getattr(hf, "rope_theta", 10000.0)))
    rtype = rp.get("rope_type", rp.get("type", "default"))
    scaling = None
    if rtype == "llama3":
        scaling = (float(rp["factor"]), float(rp["low_freq_factor"]), float(rp["high_freq_factor"]),
                   float(rp["original_max_position_embeddings"]))
    elif rtype not in ("default", None):
        raise ValueError(f"RoPE type {rtype!r} is not supported (default and llama3 are)")
    return LlamaConfig(d=d, heads=heads, kv_heads=int(getattr(hf, "num_key_value_heads", heads) or heads),
                       head_dim=hd, ffn=int(hf.intermediate_size), eps=float(hf.rms_norm_eps), theta=theta,
                       vocab=int(hf.vocab_size), layers=int(hf.num_hidden_layers), rope_scaling=scaling)


def _state(obj) -> Mapping[str, torch.Tensor]:
    if isinstance(obj, torch.nn.Module):
        return obj.state_dict()
    return obj


def _check_layer(sd: Mapping[str, torch.Tensor], cfg: LlamaConfig, prefix: str = "") -> None:
    missing = [k for k in _LAYER_KEYS if prefix + k not in sd]
    if missing:
        raise KeyError(f"layer parameters missing: {', '.join(prefix + k for k in missing)}")
    bias = [k for k in sd if k.startswith(prefix) and k.endswith("_proj.bias")]
    if bias:
        raise ValueError(f"biased projections are not W8A16 matmuls: {', '.join(bias)}")
    shapes = {
        "self_attn.q_proj.weight": (cfg.q_dim, cfg.d), "self_attn.k_proj.weight": (cfg.kv_dim, cfg.d),
        "self_attn.v_proj.weight": (cfg.kv_dim, cfg.d), "self_attn.o_proj.weight": (cfg.d, cfg.q_dim),
        "mlp.gate_proj.weight": (cfg.ffn, cfg.d), "mlp.up_proj.weight": (cfg.ffn, cfg.d),
        "mlp.down_proj.weight": (cfg.d, cfg.ffn), "input_layernorm.weight": (cfg.d,),
        "post_attention_layernorm.weight": (cfg.d,),
    }
    for k, shp in shapes.items():
        if tuple(sd[prefix + k].shape) != shp:
            raise ValueError(f"{prefix + k}: shape {tuple(sd[prefix + k].shape)}, config expects {shp}")


def layer_float(layer, cfg: LlamaConfig, prefix: str = "") -> Dict[str, torch.Tensor]:
    """A decoder layer's parameters in the reference's float layout
    (model.py:44-61 / llama_layer.py:24-31; x @ W convention, CPU float32):
    Wq{h}, Wk{k}, Wv{k} [d, hd], Wo{h} [hd, d], Wg, Wu [d, F], Wd [F, d],
    Wn1, Wn2 [d] -- the dict llama.layer_from_float and the reference's
    numpy layer both take."""
    sd = _state(layer)
    _check_layer(sd, cfg, prefix)
    g = lambda k: sd[prefix + k].detach().to("cpu", torch.float32)  # noqa: E731
    hd = cfg.head_dim
    wq, wk, wv, wo = (g(f"self_attn.{n}_proj.weight") for n in "qkvo")
    W = {"Wg": g("mlp.gate_proj.weight").t().contiguous(), "Wu": g("mlp.up_proj.weight").t().contiguous(),
         "Wd": g("mlp.down_proj.weight").t().contiguous(),
         "Wn1": g("input_layernorm.weight").clone(), "Wn2": g("post_attention_layernorm.weight").clone()}
    for h in range(cfg.heads):
        W[f"Wq{h}"] = wq[h * hd:(h + 1) * hd].t().contiguous()
        W[f"Wo{h}"] = wo[:, h * hd:(h + 1) * hd].t().contiguous()
    for k in range(cfg.kv_heads):
        W[f"Wk{k}"] = wk[k * hd:(k + 1) * hd].t().contiguous()
        W[f"Wv{k}"] = wv[k * hd:(k + 1) * hd].t().contiguous()
    return W


def layer_from_module(layer, cfg: LlamaConfig, device, tp: TP = TP(), prefix: str = "") -> LayerWeights:
    """This rank's W8A16 LayerWeights from a decoder layer module or state
    dict: the projections are fused ([q | k | v], [gate | up]), quantised per
    output channel over the full matrices on `device`, then sharded for tp
    (as llama.layer_from_float does for the reference's dict)."""
    sd = _state(layer)
    _check_layer(sd, cfg, prefix)
    dev = torch.device(device)
    g = lambda k: sd[prefix + k].detach().to(dev, torch.float32)  # noqa: E731
    Wqkv = torch.cat([g("self_attn.q_proj.weight"), g("self_attn.k_proj.weight"), g("self_attn.v_proj.weight")],
                     dim=0).t().contiguous()
    Wo = g("self_attn.o_proj.weight").t().contiguous()
    Wgu = torch.cat([g("mlp.gate_proj.weight"), g("mlp.up_proj.weight")], dim=0).t().contiguous()
    Wd = g("mlp.down_proj.weight").t().contiguous()
    g1 = g("input_layernorm.weight").half()
    g2 = g("post_attention_layernorm.weight").half()
    return _pack_layer(cfg, Wqkv, Wo, Wgu, Wd, g1, g2, tp)


def stack_from_module(model, cfg: Optional[LlamaConfig] = None, device=None, tp: TP = TP()) -> StackWeights:
    """StackWeights from a Llama causal LM (module or state dict with the
    model.embed_tokens / model.layers.<i> / model.norm / lm_head names; a
    missing lm_head.weight means tied embeddings).  cfg defaults to
    config_from_hf(model.config)."""
    if cfg is None:
        cfg = config_from_hf(model.config)
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    sd = _state(model)
    if cfg.vocab % tp.size:
        raise ValueError(f"tp={tp.size} must divide the vocabulary {cfg.vocab}")
    layers = [layer_from_module(sd, cfg, dev, tp, prefix=f"model.layers.{i}.") for i in range(cfg.layers)]
    embed = sd["model.embed_tokens.weight"].detach().to(dev, torch.float16).contiguous()
    norm = sd["model.norm.weight"].detach().to(dev, torch.float16).contiguous()
    lm = sd.get("lm_head.weight", sd["model.embed_tokens.weight"])
    vs = cfg.vocab // tp.size
    lm_shard = lm.detach()[tp.rank * vs:(tp.rank + 1) * vs].to(dev, torch.float16).contiguous()
    return StackWeights(layers, embed, norm, lm_shard, tp.rank * vs)

"""Quantised-weight files: save a W8A16 stack once, load it without the fp32
weights or the quantiser.

The reference keeps nothing between runs except the simulator's G-buffer
dump (--gout, _poc/mysim.cpp:147-155); a Llama-7B-shaped stack here is 6.5 GB
of int8 weights plus fp16 scales, embedding and lm_head, which are otherwise
re-made from fp32 on every start.

File layout (little-endian):
    8 bytes   magic b"NPUBW8\\x00\\x01"
    8 bytes   header length H (uint64)
    H bytes   UTF-8 JSON: {"config": LlamaConfig fields, "tensors": [{"name",
              "dtype", "shape", "offset", "nbytes", "crc32"}, ...]}
    then the tensors' raw bytes, each starting at a 256-byte-aligned offset
    from the start of the file.

The file holds the unsharded (tp = 1) weights.  load_stack(..., tp) cuts
each rank's shard out of them with the same rule the quantiser-side
sharding uses (llama.tp_ranges): output rows of QKV and of the interleaved
gate|up (rank r owns gate/up channels [r F/tp, (r+1) F/tp), which are rows
[2 r F/tp, 2 (r+1) F/tp) of the interleaved matrix), input columns of O and
down, vocabulary rows of the lm_head.  Scales are per output channel over the
full matrices, so the shards apply the same scales as the unsharded layer.
"""
from __future__ import annotations

import dataclasses
import json
import os
import zlib
from typing import Dict, List

import numpy as np
import torch

from .llama import TP, LayerWeights, LlamaConfig, StackWeights, tp_ranges

MAGIC = b"NPUBW8\x00\x01"
_ALIGN = 256
_DT = {torch.int8: "i1", torch.float16: "f2", torch.float32: "f4", torch.int32: "i4"}
_TD = {v: k for k, v in _DT.items()}
_LAYER_FIELDS = ("wqkv", "sqkv", "wo", "so", "wgu", "sgu", "wd", "sd", "g1", "g2")


def _layer_tensors(i: int, lw: LayerWeights) -> List[tuple]:
    return [(f"layers.{i}.{f}", getattr(lw, f)) for f in _LAYER_FIELDS]


def save_stack(path: str, cfg: LlamaConfig, w: StackWeights) -> None:
    """Write an unsharded stack (every layer holding all heads and FFN columns)."""
    for i, lw in enumerate(w.layers):
        if lw.heads != cfg.heads or lw.kv_heads != cfg.kv_heads or lw.ffn != cfg.ffn:
            raise ValueError(f"layer {i} is a tensor-parallel shard; save the unsharded (tp=1) stack")
    if w.lm_head.shape[0] != cfg.vocab or w.vocab_off != 0:
        raise ValueError("the lm_head is a vocabulary shard; save the unsharded (tp=1) stack")
    items = [("embed", w.embed), ("norm", w.norm), ("lm_head", w.lm_head)]
    for i, lw in enumerate(w.layers):
        items += _layer_tensors(i, lw)
    entries, off = [], 0
    for name, t in items:
        if t.dtype not in _DT:
            raise TypeError(f"{name}: dtype {t.dtype} is not stored")
        nb = t.numel() * t.element_size()
        entries.append({"name": name, "dtype": _DT[t.dtype], "shape": list(t.shape), "offset": off, "nbytes": nb})
        off += (nb + _ALIGN - 1) // _ALIGN * _ALIGN
    cfgd = dataclasses.asdict(cfg)
    cfgd["layers"] = len(w.layers)
    blobs = []
    for e, (_, t) in zip(entries, items):
        b = t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes() if t.numel() else b""
        e["crc32"] = zlib.crc32(b)
        blobs.append(b)
    # the data starts at the first 256-byte boundary after the header; the
    # header holds absolute offsets, so grow the reservation until it fits
    data0 = _ALIGN
    while True:
        ents = [dict(e, offset=e["offset"] + data0) for e in entries]
        hdr = json.dumps({"config": cfgd, "tensors": ents}).encode()
        if 16 + len(hdr) <= data0:
            break
        data0 = (16 + len(hdr) + _ALIGN - 1) // _ALIGN * _ALIGN
    hdr = hdr + b" " * (data0 - 16 - len(hdr))
    entries = ents
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(MAGIC)
        f.write(np.uint64(len(hdr)).tobytes())
        f.write(hdr)
        for e, b in zip(entries, blobs):
            f.seek(e["offset"])
            f.write(b)
        f.truncate(max([e["offset"] + e["nbytes"] for e in entries] + [16 + len(hdr)]))
    os.replace(tmp, path)


def read_header(path: str) -> Dict:
    with open(path, "rb") as f:
        if f.read(8) != MAGIC:
            raise ValueError(f"{path}: not a quantised-weight file")
        n = int(np.frombuffer(f.read(8), dtype=np.uint64)[0])
        return json.loads(f.read(n).decode())


def load_config(path: str) -> LlamaConfig:
    c = dict(read_header(path)["config"])
    if c.get("rope_scaling") is not None:
        c["rope_scaling"] = tuple(c["rope_scaling"])
    return LlamaConfig(**c)


def load_stack(path: str, device, tp: TP = TP(), verify: bool = True):
    """(LlamaConfig, StackWeights) of this rank, read from a save_stack file.
    verify checks every tensor's CRC-32 before it is used."""
    hdr = read_header(path)
    cfg = load_config(path)
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    dev = torch.device(device)
    ents = {e["name"]: e for e in hdr["tensors"]}

    def host(name: str) -> torch.Tensor:
        e = ents[name]
        raw = mm[e["offset"]:e["offset"] + e["nbytes"]]
        if verify and zlib.crc32(raw) != e["crc32"]:
            raise ValueError(f"{path}: {name} fails its CRC-32 check")
        return torch.from_numpy(np.array(raw).view(np.dtype(e["dtype"]))).view(_TD[e["dtype"]]).reshape(e["shape"])

    def rows(t: torch.Tensor, blocks) -> torch.Tensor:
        return torch.cat([t[r.start:r.stop] for r in blocks], dim=0)

    hq, hk, f = cfg.heads // tp.size, cfg.kv_heads // tp.size, cfg.ffn // tp.size
    if cfg.vocab % tp.size:
        raise ValueError(f"tp={tp.size} must divide the vocabulary {cfg.vocab}")
    rg = tp_ranges(cfg, tp.rank, tp.size)
    layers = []
    for i in range(cfg.layers):
        t = {k: host(f"layers.{i}.{k}") for k in _LAYER_FIELDS}
        o0, o1 = rg["o"][0].start, rg["o"][0].stop
        d0, d1 = rg["d"][0].start, rg["d"][0].stop
        r = tp.rank
        sh = {
            "wqkv": rows(t["wqkv"], rg["qkv"]), "sqkv": rows(t["sqkv"], rg["qkv"]),
            "wo": t["wo"][:, o0:o1], "so": t["so"],
            "wgu": t["wgu"][2 * r * f:2 * (r + 1) * f], "sgu": t["sgu"][2 * r * f:2 * (r + 1) * f],
            "wd": t["wd"][:, d0:d1], "sd": t["sd"], "g1": t["g1"], "g2": t["g2"],
        }
        sh = {k: v.contiguous().to(dev) for k, v in sh.items()}
        layers.append(LayerWeights(**sh, heads=hq, kv_heads=hk, ffn=f))
    vs = cfg.vocab // tp.size
    lm = host("lm_head")[tp.rank * vs:(tp.rank + 1) * vs].contiguous().to(dev)
    return cfg, StackWeights(layers, host("embed").to(dev), host("norm").to(dev), lm, tp.rank * vs)

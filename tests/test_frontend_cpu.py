"""CPU checks of the model-import side: the Llama-3 RoPE frequency table
(oracle and the library's host-side builder against the reference
compiler's own tables), the mapping of PyTorch Llama modules onto the
reference's weight layout, and the quantised-weight file format.

The module mapping is checked end to end in float64: a small Hugging Face
LlamaForCausalLM (GQA, Llama-3 RoPE scaling, random weights) against the
oracle's float64 layer (oracle/ref.py:ref_layer, model.py:115-157) fed with
frontend.layer_float's dicts and the reference's cos/sin tables."""
import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import ref

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden", "rope_tables.npz")


@pytest.mark.parametrize("name", ["llama3", "reduced", "hd128"])
def test_oracle_rope_tables_match_reference_compiler(name):
    z = np.load(GOLD)
    seq, hd, base, scaled = z[f"{name}_args"]
    rows = z[f"{name}_rows"]
    c, s = ref.rope_tables(int(seq), int(hd), float(base), llama3_scaling=bool(scaled))
    assert np.array_equal(c[rows], z[f"{name}_cos"]) and np.array_equal(s[rows], z[f"{name}_sin"])
    # rotate_half as the reference's permutation matrix (legalize.py:80-84)
    x = np.random.default_rng(0).standard_normal((3, int(hd)))
    h = int(hd) // 2
    assert np.array_equal(x @ z[f"{name}_rot"], np.concatenate([-x[:, h:], x[:, :h]], axis=1))


@pytest.mark.parametrize("hd,base,scaled", [(128, 500000.0, True), (128, 10000.0, False), (16, 10000.0, False),
                                            (64, 500000.0, True)])
def test_library_frequency_table_matches_oracle(hd, base, scaled):
    from npu_comp_b200 import _lib
    lib = _lib.load()
    out = (ctypes.c_float * (hd // 2))()
    factor = 32.0 if scaled else 0.0
    assert lib.npub_rope_llama3_freqs(ctypes.addressof(out), hd, base, factor, 1.0, 4.0, 8192.0) == 0
    want = ref.rope_freqs(hd, base, llama3_scaling=scaled).astype(np.float32)
    assert np.array_equal(np.frombuffer(out, dtype=np.float32), want)


def test_library_frequency_table_rejects_bad_arguments():
    from npu_comp_b200 import _lib
    lib = _lib.load()
    out = (ctypes.c_float * 64)()
    assert lib.npub_rope_llama3_freqs(ctypes.addressof(out), 127, 10000.0, 0.0, 1.0, 4.0, 8192.0) != 0
    assert lib.npub_rope_llama3_freqs(ctypes.addressof(out), 128, -1.0, 0.0, 1.0, 4.0, 8192.0) != 0
    assert lib.npub_rope_llama3_freqs(ctypes.addressof(out), 128, 10000.0, 32.0, 4.0, 1.0, 8192.0) != 0
    assert lib.npub_rope_llama3_freqs(None, 128, 10000.0, 0.0, 1.0, 4.0, 8192.0) != 0


def _hf_model(layers=2, seed=0):
    transformers = pytest.importorskip("transformers")
    cfg = transformers.LlamaConfig(
        hidden_size=64, intermediate_size=96, num_attention_heads=4, num_key_value_heads=2, head_dim=16,
        num_hidden_layers=layers, vocab_size=128, rms_norm_eps=1e-5, max_position_embeddings=16384,
        rope_theta=500000.0, tie_word_embeddings=False, attn_implementation="eager",
        rope_scaling={"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                      "original_max_position_embeddings": 8192})
    torch.manual_seed(seed)
    m = transformers.LlamaForCausalLM(cfg).double().eval()
    with torch.no_grad():  # norm gains away from 1 so their mapping is checked too
        for n, p in m.named_parameters():
            if n.endswith("norm.weight"):
                p.uniform_(0.8, 1.2)
    return m


def test_config_from_hf_reads_sizes_and_rope_scaling():
    from npu_comp_b200 import frontend
    m = _hf_model()
    c = frontend.config_from_hf(m.config)
    assert (c.d, c.heads, c.kv_heads, c.head_dim, c.ffn, c.vocab, c.layers) == (64, 4, 2, 16, 96, 128, 2)
    assert c.theta == 500000.0 and c.rope_scaling == (32.0, 1.0, 4.0, 8192.0) and c.eps == 1e-5


def test_hf_llama_matches_oracle_layer_on_imported_weights():
    """Logits of the HF model equal embedding -> ref_layer x L -> RMSNorm ->
    lm_head on frontend.layer_float's dicts (float64), at positions where the
    Llama-3 scaling changes the low frequencies."""
    from npu_comp_b200 import frontend
    m = _hf_model()
    c = frontend.config_from_hf(m.config)
    T = 12
    # spread positions: attention sees relative distances up to ~8000, where
    # the Llama-3 scaling changes the low frequencies
    posn = np.arange(T) * 700 + 3
    ids = torch.randint(0, c.vocab, (1, T), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        want = m(input_ids=ids, position_ids=torch.from_numpy(posn).view(1, T)).logits[0].numpy()
    sd = m.state_dict()

    def tables(scaling):
        ang = posn[:, None].astype(np.float64) * ref.rope_freqs(c.head_dim, c.theta, scaling)[None, :]
        return np.concatenate([np.cos(ang)] * 2, axis=1), np.concatenate([np.sin(ang)] * 2, axis=1)

    def logits(scaling):
        cos, sin = tables(scaling)
        x = sd["model.embed_tokens.weight"][ids[0]].numpy()
        for i in range(c.layers):
            W = {k: v.double().numpy() for k, v in frontend.layer_float(sd, c, prefix=f"model.layers.{i}.").items()}
            x = ref.ref_layer(W, x, c.heads, c.kv_heads, c.head_dim, c.eps, cos, sin)
        g = sd["model.norm.weight"].numpy()
        return (x / np.sqrt(np.mean(x * x, axis=1, keepdims=True) + c.eps) * g) @ sd["lm_head.weight"].numpy().T

    got = logits(c.rope_scaling)
    # HF evaluates the RoPE angles in float32 (its inv_freq buffer), the oracle
    # in float64: ~1e-7 apart; a wrong weight mapping is off by O(1)
    assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max()
    # without the scaling the same positions give other logits: the table matters here
    assert np.abs(logits(None) - want).max() > 1e-3 * np.abs(want).max()


def test_layer_float_rejects_bias_and_wrong_shapes():
    from npu_comp_b200 import frontend
    m = _hf_model(layers=1)
    c = frontend.config_from_hf(m.config)
    sd = dict(m.state_dict())
    sd["model.layers.0.self_attn.q_proj.bias"] = torch.zeros(64, dtype=torch.float64)
    with pytest.raises(ValueError):
        frontend.layer_float(sd, c, prefix="model.layers.0.")
    sd = dict(m.state_dict())
    del sd["model.layers.0.mlp.up_proj.weight"]
    with pytest.raises(KeyError):
        frontend.layer_float(sd, c, prefix="model.layers.0.")
    import dataclasses
    with pytest.raises(ValueError):
        frontend.layer_float(m.state_dict(), dataclasses.replace(c, ffn=64), prefix="model.layers.0.")
    with pytest.raises(ValueError):
        frontend.quantize_linear(torch.nn.Linear(4, 4, bias=True))


def _cpu_stack(cfg, seed=0):
    from npu_comp_b200 import llama
    g = torch.Generator().manual_seed(seed)

    def i8(*s):
        return torch.randint(-127, 128, s, generator=g, dtype=torch.int8)

    def f16(*s):
        return torch.randn(s, generator=g).half()

    qkv = cfg.q_dim + 2 * cfg.kv_dim
    layers = [llama.LayerWeights(i8(qkv, cfg.d), f16(qkv), i8(cfg.d, cfg.q_dim), f16(cfg.d), i8(2 * cfg.ffn, cfg.d),
                                 f16(2 * cfg.ffn), i8(cfg.d, cfg.ffn), f16(cfg.d), f16(cfg.d), f16(cfg.d),
                                 cfg.heads, cfg.kv_heads, cfg.ffn) for _ in range(cfg.layers)]
    return llama.StackWeights(layers, f16(cfg.vocab, cfg.d), f16(cfg.d), f16(cfg.vocab, cfg.d), 0)


def test_weight_file_roundtrip_and_tp_shards(tmp_path):
    from npu_comp_b200 import checkpoint, llama
    cfg = llama.LlamaConfig(d=64, heads=4, kv_heads=2, head_dim=16, ffn=96, vocab=128, layers=2, theta=500000.0,
                            rope_scaling=(32.0, 1.0, 4.0, 8192.0))
    w = _cpu_stack(cfg)
    path = str(tmp_path / "stack.npubw")
    checkpoint.save_stack(path, cfg, w)
    c2, w2 = checkpoint.load_stack(path, "cpu")
    assert c2 == cfg
    for a, b in zip(w.layers, w2.layers):
        for f in ("wqkv", "sqkv", "wo", "so", "wgu", "sgu", "wd", "sd", "g1", "g2"):
            assert torch.equal(getattr(a, f), getattr(b, f)), f
    for f in ("embed", "norm", "lm_head"):
        assert torch.equal(getattr(w, f), getattr(w2, f))
    # tp = 2 shards put back together give the unsharded tensors
    sh = [checkpoint.load_stack(path, "cpu", tp=llama.TP(r, 2))[1] for r in range(2)]
    for li, full in enumerate(w.layers):
        a, b = sh[0].layers[li], sh[1].layers[li]
        hd, hq, hk = cfg.head_dim, cfg.heads // 2, cfg.kv_heads // 2
        q = torch.cat([a.wqkv[:hq * hd], b.wqkv[:hq * hd]])
        k = torch.cat([a.wqkv[hq * hd:(hq + hk) * hd], b.wqkv[hq * hd:(hq + hk) * hd]])
        v = torch.cat([a.wqkv[(hq + hk) * hd:], b.wqkv[(hq + hk) * hd:]])
        assert torch.equal(torch.cat([q, k, v]), full.wqkv)
        assert torch.equal(torch.cat([a.wo, b.wo], dim=1), full.wo) and torch.equal(a.so, full.so)
        assert torch.equal(torch.cat([a.wgu, b.wgu]), full.wgu) and torch.equal(torch.cat([a.sgu, b.sgu]), full.sgu)
        assert torch.equal(torch.cat([a.wd, b.wd], dim=1), full.wd)
        assert (a.heads, a.kv_heads, a.ffn) == (hq, hk, cfg.ffn // 2)
    assert torch.equal(torch.cat([sh[0].lm_head, sh[1].lm_head]), w.lm_head) and sh[1].vocab_off == cfg.vocab // 2


def test_weight_file_detects_corruption_and_refuses_shards(tmp_path):
    from npu_comp_b200 import checkpoint, llama
    cfg = llama.LlamaConfig(d=64, heads=4, kv_heads=2, head_dim=16, ffn=96, vocab=128, layers=1)
    w = _cpu_stack(cfg, seed=3)
    path = str(tmp_path / "s.npubw")
    checkpoint.save_stack(path, cfg, w)
    hdr = checkpoint.read_header(path)
    e = [t for t in hdr["tensors"] if t["name"] == "layers.0.wd"][0]
    assert e["offset"] % 256 == 0
    with open(path, "r+b") as f:
        f.seek(e["offset"] + 5)
        b = f.read(1)
        f.seek(e["offset"] + 5)
        f.write(bytes([b[0] ^ 1]))
    with pytest.raises(ValueError, match="CRC"):
        checkpoint.load_stack(path, "cpu")
    sh = checkpoint.load_stack(str(tmp_path / "s.npubw"), "cpu", tp=llama.TP(0, 2), verify=False)[1]
    with pytest.raises(ValueError):
        checkpoint.save_stack(str(tmp_path / "t.npubw"), cfg, sh)
    with open(str(tmp_path / "junk"), "wb") as f:
        f.write(b"not a weight file")
    with pytest.raises(ValueError):
        checkpoint.read_header(str(tmp_path / "junk"))

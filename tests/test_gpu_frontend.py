"""Model import and Llama-3 RoPE on the GPU against the oracle.

  * RoPE with a frequency table (npub_rope_freqs, the prompt and decode
    RoPE + KV-cache kernels) on the Llama 3.2 3B head layout (24 q / 8 kv
    heads of 128, base 500000, Llama-3 scaling: model.py:20-21,
    legalize.py:50-76) at positions up to ~8000, against the oracle's float64
    rotation with the reference's table;
  * a Llama 3.2 3B-shaped layer (d 3072, FFN 8192), prefill and a decode
    step, against oracle/ref.py's float64 layer (model.py:115-157) on the
    same quantised weights with the scaled table;
  * a PyTorch (Hugging Face) Llama imported through npu_comp_b200.frontend:
    layer output against the oracle on the dequantised imported weights,
    and the stack's prefill logits against the float64 stack;
  * a quantised-weight file written and read back drives the stack to the
    same tokens as the weights it was written from.

Tolerance: normwise relative error <= 1e-2 (TOL).
"""
import numpy as np
import pytest
import torch

from npu_comp_b200 import checkpoint, frontend, llama, npu
from oracle import ref

pytestmark = pytest.mark.gpu
TOL = 1e-2
C3B = llama.LLAMA_3_2_3B


def _layer_numpy(w):
    return {n: getattr(w, n).cpu().numpy() for n in ("wqkv", "sqkv", "wo", "so", "wgu", "sgu", "wd", "sd", "g1",
                                                      "g2")}


def test_rope_table_matches_oracle_at_long_positions(cuda_device):
    hd, H = 128, C3B.heads + C3B.kv_heads
    f = ref.rope_freqs(hd, C3B.theta, llama3_scaling=True)
    tab = llama.rope_inv_freq(C3B, cuda_device)
    assert np.array_equal(tab.cpu().numpy(), f.astype(np.float32))
    g = torch.Generator(device=cuda_device).manual_seed(3)
    T = 96
    x = torch.randn((T, H * hd), generator=g, device=cuda_device).half()
    pos = torch.arange(T, device=cuda_device, dtype=torch.int32) * 83 + 17          # up to ~7900
    y = npu.rope(x.clone(), H, hd, positions=pos, inv_freq=tab).float().cpu().numpy()
    want = ref._rope64(x.float().cpu().numpy().astype(np.float64), H, hd, pos.cpu().numpy(), C3B.theta, f)
    assert ref.rel_err(y, want) <= TOL
    # the unscaled frequencies give a clearly different rotation at these positions
    y0 = npu.rope(x.clone(), H, hd, positions=pos, theta=C3B.theta).float().cpu().numpy()
    assert ref.rel_err(y0, want) > 10 * TOL


def test_rope_kv_kernels_with_table_match_rope(cuda_device):
    hd, hq, hk = 128, C3B.heads, C3B.kv_heads
    tab = llama.rope_inv_freq(C3B, cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(4)
    B, cap = 6, 8200
    qkv = torch.randn((B, (hq + 2 * hk) * hd), generator=g, device=cuda_device).half()
    pos = torch.tensor([0, 1, 4095, 4096, 8000, 8191], dtype=torch.int32, device=cuda_device)
    kc = torch.zeros((B, hk, cap, hd), dtype=torch.float16, device=cuda_device)
    vc = torch.zeros_like(kc)
    lens = torch.zeros((B,), dtype=torch.int32, device=cuda_device)
    a = qkv.clone()
    npu.rope_kv_append(a, hq, hk, hd, pos, kc, vc, lens=lens, inv_freq=tab)
    b = qkv.clone()
    npu.rope(b, hq + hk, hd, positions=pos, inv_freq=tab)
    assert torch.equal(a, b)
    assert torch.equal(lens, pos + 1)
    for i in range(B):
        p = int(pos[i])
        assert torch.equal(kc[i, :, p], b[i, hq * hd:(hq + hk) * hd].view(hk, hd))
        assert torch.equal(vc[i, :, p], b[i, (hq + hk) * hd:].view(hk, hd))
    # prompt form: 2 sequences of 3 rows
    kc2 = torch.zeros((2, hk, cap, hd), dtype=torch.float16, device=cuda_device)
    vc2 = torch.zeros_like(kc2)
    c = qkv.clone()
    npu.rope_kv_store(c, hq, hk, hd, pos, kc2, vc2, tokens_per_seq=3, inv_freq=tab)
    assert torch.equal(c, b)
    for i in range(B):
        assert torch.equal(kc2[i // 3, :, int(pos[i])], b[i, hq * hd:(hq + hk) * hd].view(hk, hd))


def test_llama_3_2_3b_layer_prefill_and_decode_against_oracle(cuda_device):
    w = llama.make_layer(C3B, seed=11, device=cuda_device)
    L = _layer_numpy(w)
    f = ref.rope_freqs(C3B.head_dim, C3B.theta, llama3_scaling=True)
    g = torch.Generator(device=cuda_device).manual_seed(5)
    T = 128
    x = torch.randn((T, C3B.d), generator=g, device=cuda_device).half()
    positions = torch.arange(T, device=cuda_device, dtype=torch.int32) * 61        # relative distances to ~7700
    y = llama.layer_prefill(x, w, C3B, positions=positions).float().cpu().numpy()
    yr = ref.ref_layer_q(L, x.float().cpu().numpy(), C3B.heads, C3B.kv_heads, C3B.head_dim, C3B.eps, C3B.theta,
                         positions=positions.cpu().numpy(), inv_freq=f)
    assert ref.rel_err(y, yr) <= TOL
    # one decode step for 4 sequences over a cache of random (already rotated) keys
    B, ctx = 4, 1000
    kc = torch.randn((B, C3B.kv_heads, ctx + 8, C3B.head_dim), generator=g, device=cuda_device).half()
    vc = torch.randn((B, C3B.kv_heads, ctx + 8, C3B.head_dim), generator=g, device=cuda_device).half()
    xd = torch.randn((B, C3B.d), generator=g, device=cuda_device).half()
    pos = torch.tensor([ctx, 999, 500, 3], dtype=torch.int32, device=cuda_device)
    kh, vh = kc.cpu().numpy(), vc.cpu().numpy()
    yd = llama.layer_decode(xd, w, C3B, kc, vc, pos, ctx_max=ctx + 1).float().cpu().numpy()
    ydr = ref.ref_decode_layer_q(L, xd.float().cpu().numpy(), kh, vh, pos.cpu().numpy(), C3B.heads, C3B.kv_heads,
                                 C3B.head_dim, C3B.eps, C3B.theta, inv_freq=f)
    assert ref.rel_err(yd, ydr) <= TOL


def _hf_model(seed=0):
    transformers = pytest.importorskip("transformers")
    cfg = transformers.LlamaConfig(
        hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
        num_hidden_layers=2, vocab_size=512, rms_norm_eps=1e-5, max_position_embeddings=16384,
        rope_theta=500000.0, tie_word_embeddings=False, attn_implementation="eager",
        rope_scaling={"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                      "original_max_position_embeddings": 8192})
    torch.manual_seed(seed)
    m = transformers.LlamaForCausalLM(cfg).eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            if n.endswith("norm.weight"):
                p.uniform_(0.8, 1.2)
            elif p.dim() == 2 and "embed" not in n:
                p.normal_(0.0, 0.05)
    return m


def test_imported_hf_layer_against_oracle_and_module(cuda_device):
    m = _hf_model()
    c = frontend.config_from_hf(m.config)
    sd = m.state_dict()
    w = frontend.layer_from_module(sd, c, cuda_device, prefix="model.layers.0.")
    T = 64
    g = torch.Generator(device=cuda_device).manual_seed(6)
    x = torch.randn((T, c.d), generator=g, device=cuda_device).half()
    posn = torch.arange(T, device=cuda_device, dtype=torch.int32) * 120
    y = llama.layer_prefill(x, w, c, positions=posn).float().cpu().numpy()
    # oracle on the dequantised imported weights, with the reference's scaled table
    f = ref.rope_freqs(c.head_dim, c.theta, llama3_scaling=c.rope_scaling)
    yr = ref.ref_layer_q(_layer_numpy(w), x.float().cpu().numpy(), c.heads, c.kv_heads, c.head_dim, c.eps, c.theta,
                         positions=posn.cpu().numpy(), inv_freq=f)
    assert ref.rel_err(y, yr) <= TOL
    # and the float module itself (its weights unquantised): int8 rounding stays small
    layer = m.model.layers[0].double()
    rot = m.model.rotary_emb
    xh = x.double().cpu().view(1, T, c.d)
    ph = posn.long().cpu().view(1, T)
    with torch.no_grad():
        cos, sin = rot(xh, ph)
        mask = torch.full((T, T), float("-inf"), dtype=torch.float64).triu(1).view(1, 1, T, T)
        out = layer(xh, attention_mask=mask, position_ids=ph, position_embeddings=(cos.double(), sin.double()))
    yh = (out[0] if isinstance(out, tuple) else out)[0].numpy()
    assert ref.rel_err(y, yh) <= 3 * TOL


def test_imported_hf_stack_prefill_logits_against_oracle(cuda_device):
    m = _hf_model(seed=1)
    c = frontend.config_from_hf(m.config)
    sw = frontend.stack_from_module(m, c, cuda_device)
    B, T = 2, 16
    prompts = torch.randint(0, c.vocab, (B, T), generator=torch.Generator().manual_seed(2), dtype=torch.int32)
    st = llama.LlamaStack(c, sw, B, T, 2, cuda_device, use_graph=False)
    st.prefill(prompts.to(cuda_device))
    got = st.sc.bufs["logits"].float().cpu().numpy()
    layers = [_layer_numpy(lw) for lw in sw.layers]
    want = ref.ref_stack_logits(layers, sw.embed.cpu().numpy(), sw.norm.cpu().numpy(), sw.lm_head.cpu().numpy(),
                                prompts.numpy(), c.heads, c.kv_heads, c.head_dim, c.eps, c.theta,
                                rows=np.array([T - 1]), inv_freq=ref.rope_freqs(c.head_dim, c.theta,
                                                                                c.rope_scaling))[:, 0]
    assert ref.rel_err(got, want) <= TOL


def test_weight_file_drives_the_stack_to_the_same_tokens(cuda_device, tmp_path):
    cfg = llama.LlamaConfig(d=1024, heads=8, kv_heads=4, head_dim=128, ffn=2816, vocab=4096, layers=2)
    sw = llama.make_stack(cfg, seed=5, device=cuda_device)
    path = str(tmp_path / "w.npubw")
    checkpoint.save_stack(path, cfg, sw)
    c2, sw2 = checkpoint.load_stack(path, cuda_device)
    assert c2 == cfg
    B, T = 3, 32
    prompts = torch.randint(0, cfg.vocab, (B, T), generator=torch.Generator().manual_seed(9),
                            dtype=torch.int32).to(cuda_device)
    toks = []
    for w in (sw, sw2):
        st = llama.LlamaStack(cfg, w, B, T, 4, cuda_device)
        st.prefill(prompts)
        st.decode(4, record=True)
        toks.append(torch.stack(st.tokens).cpu())
        st.release()
    assert npu.device_error() == 0
    assert torch.equal(toks[0], toks[1])

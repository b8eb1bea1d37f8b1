"""The Llama layer and stack at the benchmarked sizes on the GPU against the
float64 oracle (oracle/ref.py: ref_layer_q, ref_decode_layer_q,
ref_stack_logits -- model.py:115-157 restated over the build's quantised,
fused weights, which apply q * s exactly).

  * one Llama-7B layer, prefill of a 2048-token prompt (x ~N(0,1), weights
    ~N(0,0.02) quantised per output channel): every row;
  * one decode step of that layer for 64 sequences over a 4096-token fp16 KV
    cache ~N(0,1);
  * the decoder stack (embedding, W8A16 layers, final RMSNorm, fp16 lm_head):
    a 2-layer Llama-7B-shaped stack, prefill logits and 4 graph-replayed
    greedy decode steps, and the 32-layer stack's prefill logits.

Tolerance: normwise relative error max|got - ref| / max|ref| <= 1e-2 (TOL, the
reference's convention); the mean absolute error is printed and bounded by
TOL times the mean |ref|.
"""
import numpy as np
import pytest
import torch

from npu_comp_b200 import llama
from oracle import ref

pytestmark = pytest.mark.gpu
TOL = 1e-2
CFG = llama.LLAMA_7B


def layer_numpy(w: llama.LayerWeights) -> dict:
    """One layer's weights on the host, in the layout ref_layer_q takes."""
    names = ("wqkv", "sqkv", "wo", "so", "wgu", "sgu", "wd", "sd", "g1", "g2")
    return {n: getattr(w, n).cpu().numpy() for n in names}


def report(name, got, want):
    """Normwise relative error and mean absolute error relative to the mean |ref|."""
    e = ref.rel_err(got, want)
    mae = float(np.abs(np.asarray(got, np.float64) - want).mean())
    rmae = mae / float(np.abs(want).mean())
    print(f"{name}: rel {e:.3e}, mean abs {mae:.3e} ({rmae:.2e} of mean |ref|)")
    return e, rmae


def test_layer_prefill_t2048_against_oracle(cuda_device):
    w = llama.make_layer(CFG, seed=0, device=cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(7)
    x = torch.randn((2048, CFG.d), generator=g, device=cuda_device).half()
    y = llama.layer_prefill(x, w, CFG).float().cpu().numpy()
    yr = ref.ref_layer_q(layer_numpy(w), x.float().cpu().numpy(), CFG.heads, CFG.kv_heads, CFG.head_dim, CFG.eps,
                         CFG.theta)
    e, mae = report("layer T=2048", y, yr)
    assert e <= TOL
    assert mae <= TOL
    # every row on its own, the last (longest-context) rows included
    rows = np.abs(y - yr).max(axis=1) / np.abs(yr).max(axis=1)
    assert rows.max() <= 2 * TOL, (int(rows.argmax()), float(rows.max()))
    assert rows[-64:].max() <= 2 * TOL


def test_layer_decode_b64_kv4096_against_oracle(cuda_device):
    B, ctx = 64, 4096
    w = llama.make_layer(CFG, seed=0, device=cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(8)
    kc = torch.randn((B, CFG.kv_heads, ctx + 8, CFG.head_dim), generator=g, device=cuda_device).half()
    vc = torch.randn((B, CFG.kv_heads, ctx + 8, CFG.head_dim), generator=g, device=cuda_device).half()
    x = torch.randn((B, CFG.d), generator=g, device=cuda_device).half()
    pos = torch.full((B,), ctx, dtype=torch.int32, device=cuda_device)
    kh, vh = kc.cpu().numpy(), vc.cpu().numpy()   # positions < ctx are left as they are
    y = llama.layer_decode(x, w, CFG, kc, vc, pos, ctx_max=ctx + 1).float().cpu().numpy()
    yr = ref.ref_decode_layer_q(layer_numpy(w), x.float().cpu().numpy(), kh, vh, np.full(B, ctx), CFG.heads,
                                CFG.kv_heads, CFG.head_dim, CFG.eps, CFG.theta)
    e, mae = report("decode B=64 KV=4096", y, yr)
    assert e <= TOL
    assert mae <= TOL
    rows = np.abs(y - yr).max(axis=1) / np.abs(yr).max(axis=1)
    assert rows.max() <= 2 * TOL


def _stack_oracle(w, prompts_h, gen_h, rows):
    """Oracle logits [B, len(rows), vocab] of each sequence over its prompt
    followed by the generated tokens; layer weights are fetched one at a time."""
    toks = np.concatenate([prompts_h, gen_h], axis=1) if gen_h is not None else prompts_h
    layers = (layer_numpy(lw) for lw in w.layers)
    return ref.ref_stack_logits(layers, w.embed.cpu().numpy(), w.norm.cpu().numpy(), w.lm_head.cpu().numpy(), toks,
                                CFG.heads, CFG.kv_heads, CFG.head_dim, CFG.eps, CFG.theta, rows=rows)


def test_stack_2_layers_prefill_and_graph_decode_against_oracle(cuda_device):
    """Llama-7B-shaped stack (2 layers, vocab 32000): the prefill logits and the
    logits of 4 greedy decode steps replayed from the CUDA graph, against the
    float64 stack over the prompt followed by the tokens the GPU chose."""
    B, T, S = 2, 48, 4
    w = llama.make_stack(CFG, seed=1, device=cuda_device, layers=2)
    g = torch.Generator(device=cuda_device).manual_seed(9)
    prompts = torch.randint(0, CFG.vocab, (B, T), generator=g, device=cuda_device, dtype=torch.int32)
    st = llama.LlamaStack(CFG, w, B, T, S, cuda_device, use_graph=True)
    logits = [None] * (S + 1)
    st.prefill(prompts)
    logits[0] = st.sc.bufs["logits"].float().cpu().numpy()
    for s in range(S):
        st.decode(1, record=True)
        logits[s + 1] = st.sc.bufs["logits"].float().cpu().numpy()
    assert st.graph is not None
    gen = torch.stack(st.tokens[:S], dim=1).cpu().numpy()   # tokens fed to decode steps 1..S
    want = _stack_oracle(w, prompts.cpu().numpy(), gen, rows=np.arange(T - 1, T + S))
    for s in range(S + 1):
        e, mae = report(f"stack2 step {s}", logits[s], want[:, s])
        assert e <= TOL, (s, e)
        assert mae <= TOL
    # the GPU's greedy choice is the oracle's argmax wherever the top two logits differ clearly
    for s in range(S):
        for b in range(B):
            top2 = np.sort(want[b, s])[-2:]
            if top2[1] - top2[0] > 2e-2 * np.abs(want[b, s]).max():
                assert gen[b, s] == int(np.argmax(want[b, s]))
    st.release()


def test_stack_32_layers_prefill_logits_against_oracle(cuda_device):
    """The benchmarked 32-layer Llama-7B W8A16 stack: prefill logits of the last
    prompt position for 2 prompts, against the float64 stack."""
    B, T = 2, 16
    w = llama.make_stack(CFG, seed=0, device=cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(10)
    prompts = torch.randint(0, CFG.vocab, (B, T), generator=g, device=cuda_device, dtype=torch.int32)
    st = llama.LlamaStack(CFG, w, B, T, 1, cuda_device, use_graph=False)
    st.prefill(prompts)
    got = st.sc.bufs["logits"].float().cpu().numpy()
    want = _stack_oracle(w, prompts.cpu().numpy(), None, rows=np.array([T - 1]))[:, 0]
    e, mae = report("stack32 prefill", got, want)
    assert e <= TOL
    assert mae <= TOL

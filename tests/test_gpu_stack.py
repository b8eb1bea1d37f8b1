"""The decoder stack (embedding -> W8A16 layers -> lm_head -> greedy argmax) on
the GPU: graph-replayed decode equals eager decode, and the logits of a decode
step equal those of a prefill over the longer sequence.
Tolerance: normwise relative error <= 1e-2 (TOL)."""
import pytest
import torch

from npu_comp_b200 import llama

pytestmark = pytest.mark.gpu
TOL = 1e-2
CFG = llama.LlamaConfig(d=512, heads=4, kv_heads=2, head_dim=128, ffn=1376, eps=1e-5, theta=10000.0, vocab=1024,
                        layers=2)


def _prompts(dev, B, T, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    return torch.randint(0, CFG.vocab, (B, T), generator=g, device=dev, dtype=torch.int32)


def test_graph_decode_equals_eager_decode(cuda_device):
    w = llama.make_stack(CFG, seed=3, device=cuda_device)
    prompts = _prompts(cuda_device, 3, 40)
    a = llama.LlamaStack(CFG, w, 3, 40, 6, cuda_device, use_graph=True)
    b = llama.LlamaStack(CFG, w, 3, 40, 6, cuda_device, use_graph=False)
    a.prefill(prompts)
    a.decode(6, record=True)
    b.prefill(prompts)
    b.decode(6, record=True)
    assert a.graph is not None
    ta, tb = torch.stack(a.tokens), torch.stack(b.tokens)
    assert ta.shape == (7, 3)
    assert torch.equal(ta, tb)
    assert int(a.pos[0]) == 46 and int(b.pos[0]) == 46


def test_decode_logits_match_longer_prefill(cuda_device):
    w = llama.make_stack(CFG, seed=5, device=cuda_device)
    B, T = 2, 33
    prompts = _prompts(cuda_device, B, T, seed=1)
    s = llama.LlamaStack(CFG, w, B, T, 1, cuda_device, use_graph=False)
    first = s.prefill(prompts).clone()
    s.decode(1)
    dec_logits = s.sc.get("logits", (B, CFG.vocab), device=cuda_device).float().clone()
    longer = torch.cat([prompts, first.view(B, 1)], dim=1).contiguous()
    s2 = llama.LlamaStack(CFG, w, B, T + 1, 1, cuda_device, use_graph=False)
    s2.prefill(longer)
    pre_logits = s2.sc.get("logits", (B, CFG.vocab), device=cuda_device).float()
    e = ((dec_logits - pre_logits).abs().max() / pre_logits.abs().max()).item()
    assert e <= TOL, e

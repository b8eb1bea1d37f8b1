"""Attention on the GPU against the oracle: causal GQA prefill (tcgen05 GEMMs +
softmax), decode over a KV cache, and the KV-cache append.
Tolerance: normwise relative error <= 1e-2 (TOL)."""
import math

import numpy as np
import pytest
import torch

import npu_comp_b200 as nb
from oracle import ref

pytestmark = pytest.mark.gpu
TOL = 1e-2


def dev(a, d):
    return torch.from_numpy(np.ascontiguousarray(a)).to(d)


@pytest.mark.parametrize("B,T,H,KV,hd,causal", [(1, 256, 2, 2, 128, True), (2, 200, 4, 2, 64, True),
                                                 (1, 8, 4, 2, 16, True), (1, 130, 2, 1, 128, False),
                                                 (3, 77, 2, 2, 32, True)])
def test_prefill_attention(cuda_device, rng, B, T, H, KV, hd, causal):
    q = rng.standard_normal((B * T, H * hd)).astype(np.float16)
    k = rng.standard_normal((B * T, KV * hd)).astype(np.float16)
    v = rng.standard_normal((B * T, KV * hd)).astype(np.float16)
    o = nb.attention(dev(q, cuda_device), dev(k, cuda_device), dev(v, cuda_device), H, KV, head_dim=hd,
                     batch=B, causal=causal).float().cpu().numpy()
    for b in range(B):
        sl = slice(b * T, (b + 1) * T)
        exp = ref.attention_ref(q[sl], k[sl], v[sl], H, KV, hd, causal)
        assert ref.rel_err(o[sl], exp) <= TOL


def test_prefill_attention_full_size(cuda_device):
    """32 heads x 2048 tokens x 128: sampled heads against the float64 oracle."""
    g = torch.Generator(device=cuda_device).manual_seed(11)
    T, H, hd = 2048, 32, 128
    qkv = torch.randn((T, 3 * H * hd), generator=g, device=cuda_device).half()
    q, k, v = qkv[:, :H * hd], qkv[:, H * hd:2 * H * hd], qkv[:, 2 * H * hd:]
    o = nb.attention(q, k, v, H, H).float().cpu().numpy()
    qn, kn, vn = (t.cpu().numpy() for t in (q, k, v))
    for h in (0, 17, 31):
        sl = slice(h * hd, (h + 1) * hd)
        exp = ref.attention_ref(qn[:, sl], kn[:, sl], vn[:, sl], 1, 1, hd, True)
        assert ref.rel_err(o[:, sl], exp) <= TOL


def test_attention_reference_example(cuda_device, examples):
    """The reference's single-head causal attention example (test_attention.py)."""
    X, Wq, Wk, Wv, Wo = (examples[f"attention_{k}"].astype(np.float16) for k in ("X", "Wq", "Wk", "Wv", "Wo"))
    x = dev(X, cuda_device)
    q = nb.matmul(x, dev(Wq.T, cuda_device))
    k = nb.matmul(x, dev(Wk.T, cuda_device))
    v = nb.matmul(x, dev(Wv.T, cuda_device))
    ctx = nb.attention(q, k, v, 1, 1, head_dim=Wq.shape[1])
    out = nb.matmul(ctx, dev(Wo.T, cuda_device)).float().cpu().numpy()
    assert np.abs(out - examples["attention_npu"]).max() < 2e-2  # test_attention.py:75
    assert ref.rel_err(out, examples["attention_ref"]) <= TOL


@pytest.mark.parametrize("B,H,KV,ctx,cap", [(4, 8, 4, 300, 320), (2, 4, 4, 4096, 4100), (3, 2, 1, 1, 8),
                                            (8, 32, 32, 1000, 1024), (2, 16, 2, 777, 800), (2, 6, 2, 200, 256),
                                            (64, 8, 8, 128, 128)])
def test_decode_attention(cuda_device, rng, B, H, KV, ctx, cap):
    hd = 128
    q = rng.standard_normal((B, H * hd)).astype(np.float16)
    kc = rng.standard_normal((B, KV, cap, hd)).astype(np.float16)
    vc = rng.standard_normal((B, KV, cap, hd)).astype(np.float16)
    lens = rng.integers(1, ctx + 1, B).astype(np.int32)
    o = nb.attention_decode(dev(q, cuda_device), dev(kc, cuda_device), dev(vc, cuda_device), heads=H, kv_heads=KV,
                            lens=dev(lens, cuda_device), ctx_len=ctx).float().cpu().numpy()
    assert ref.rel_err(o, ref.decode_attention_ref(q, kc, vc, lens, H, KV, hd)) <= TOL


@pytest.mark.parametrize("B,H,KV,ctx,cap,lens", [
    (4, 32, 32, 4096, 4096, [1, 1, 1, 1]),          # persistent: far fewer stages than CTAs
    (5, 8, 8, 300, 320, [0, 300, 0, 64, 65]),       # persistent: sequences without keys give zeros
    (1, 32, 32, 16384, 16384, [16384]),             # persistent: each item cut into ~9 pieces
    (8, 64, 8, 4000, 4000, [4000, 1, 64, 65, 3999, 128, 2, 700]),  # persistent, groups of 8
    (1, 32, 8, 32768, 32768, [32768]),              # few items: context splits + combine
    (2, 64, 8, 20000, 20000, [20000, 1]),           # the same, groups of 8
    (520, 8, 8, 70, 72, None),                      # many items: one CTA per (sequence, kv head)
    (900, 8, 1, 100, 128, "with-empty"),            # the same with groups of 8 and empty sequences
    (32, 24, 8, 1100, 1104, None),                  # groups of 3 (Llama-3.2-3B), persistent
    (6, 48, 8, 900, 904, None),                     # groups of 6, persistent
    (120, 40, 8, 50, 64, None),                     # groups of 5, one CTA per item
    (3, 21, 3, 2000, 2000, None),                   # groups of 7, context splits
    (32, 32, 32, 1088, 1088, None),                 # one CTA per item, the last partial wave in pieces
    (120, 32, 8, 700, 704, "tail-edge"),            # the same, groups of 4, tail items with 0, 1, 130 keys
    (152, 64, 8, 600, 600, None),                   # the same, groups of 8
])
def test_decode_attention_work_split(cuda_device, rng, B, H, KV, ctx, cap, lens):
    """The three schedules of the streaming kernel (persistent grid over the
    stage list with items cut between CTAs, CTAs without stages and sequences
    without keys; context splits and a combine pass; one CTA per item, the
    items past the last whole wave cut in pieces merged by the last to
    finish) match the oracle, and a second call on new data (the piece flags
    and counts left zero) does too."""
    hd = 128
    if lens is None:
        lens = rng.integers(1, ctx + 1, B)
    elif lens == "with-empty":
        lens = rng.integers(1, ctx + 1, B) * (rng.random(B) > 0.1)
    elif lens == "tail-edge":
        lens = rng.integers(1, ctx + 1, B)
        lens[-3:] = [0, 1, 130]
    lens = np.asarray(lens, dtype=np.int32)
    kc = torch.empty((B, KV, cap, hd), dtype=torch.float16, device=cuda_device)
    vc = torch.empty_like(kc)
    for rep in range(2):
        q = rng.standard_normal((B, H * hd)).astype(np.float16)
        kh = rng.standard_normal((B, KV, cap, hd)).astype(np.float16)
        vh = rng.standard_normal((B, KV, cap, hd)).astype(np.float16)
        kc.copy_(torch.from_numpy(kh))
        vc.copy_(torch.from_numpy(vh))
        o = nb.attention_decode(dev(q, cuda_device), kc, vc, heads=H, kv_heads=KV, lens=dev(lens, cuda_device),
                                ctx_len=ctx).float().cpu().numpy()
        assert nb.npu.device_error() == 0
        live = lens > 0
        assert not o[~live].any()
        r = ref.decode_attention_ref(q[live], kh[live], vh[live], lens[live], H, KV, hd)
        assert ref.rel_err(o[live], r) <= TOL


def test_decode_matches_last_prefill_row(cuda_device, rng):
    """Decode of token T over a cache of T keys == row T of causal prefill over T+1 tokens."""
    T, H, hd = 97, 4, 128
    q = rng.standard_normal((T + 1, H * hd)).astype(np.float16)
    k = rng.standard_normal((T + 1, H * hd)).astype(np.float16)
    v = rng.standard_normal((T + 1, H * hd)).astype(np.float16)
    full = nb.attention(dev(q, cuda_device), dev(k, cuda_device), dev(v, cuda_device), H, H).float()
    kc = torch.zeros((1, H, 128, hd), dtype=torch.float16, device=cuda_device)
    vc = torch.zeros_like(kc)
    for t in range(T + 1):
        nb.kv_append(dev(k[t:t + 1], cuda_device), dev(v[t:t + 1], cuda_device), kc, vc, pos0=t)
    kv_ref = k.reshape(T + 1, H, hd).transpose(1, 0, 2)
    assert np.array_equal(kc[0, :, :T + 1].cpu().numpy(), kv_ref)
    lens = torch.tensor([T + 1], dtype=torch.int32, device=cuda_device)
    o = nb.attention_decode(dev(q[T:T + 1], cuda_device), kc, vc, heads=H, lens=lens, ctx_len=T + 1).float()
    e = ((o[0] - full[T]).abs().max() / full[T].abs().max()).item()
    assert e <= TOL


@pytest.mark.parametrize("B,T,H,KV,hd,cap", [(3, 37, 8, 4, 128, 50), (2, 64, 32, 32, 128, 80), (4, 9, 6, 2, 64, 9),
                                              (1, 5, 40, 8, 128, 5)])
def test_rope_kv_store_matches_separate_ops(cuda_device, B, T, H, KV, hd, cap):
    """The fused prefill op equals rope() on q|k heads of every prompt row, then
    a strided copy of the rotated k and the v heads into cache slots
    [b, h, positions[r]], bit for bit; rows whose position is outside
    [0, cap) are rotated but leave the caches alone."""
    g = torch.Generator(device=cuda_device).manual_seed(B * T + H)
    qkv = torch.randn((B * T, (H + 2 * KV) * hd), generator=g, device=cuda_device).half()
    pos = torch.arange(T, device=cuda_device, dtype=torch.int32).repeat(B) + 2
    pos[T - 1] = cap + 3  # first prompt's last row: out of range, not stored
    kc = torch.randn((B, KV, cap, hd), generator=g, device=cuda_device).half()
    vc = torch.randn_like(kc)
    q1, kc1, vc1 = qkv.clone(), kc.clone(), vc.clone()
    nb.rope(q1, H + KV, hd, positions=pos, theta=10000.0)
    k1 = q1[:, H * hd:(H + KV) * hd].reshape(B, T, KV, hd)
    v1 = q1[:, (H + KV) * hd:].reshape(B, T, KV, hd)
    for b in range(B):
        for t in range(T):
            p = int(pos[b * T + t])
            if 0 <= p < cap:
                kc1[b, :, p] = k1[b, t]
                vc1[b, :, p] = v1[b, t]
    nb.rope_kv_store(qkv, H, KV, hd, pos, kc, vc, tokens_per_seq=T, theta=10000.0)
    assert torch.equal(qkv, q1)
    assert torch.equal(kc, kc1) and torch.equal(vc, vc1)


@pytest.mark.parametrize("B,H,KV,hd,cap", [(5, 8, 4, 128, 40), (3, 32, 32, 128, 300), (2, 6, 2, 64, 17)])
def test_rope_kv_append_matches_separate_ops(cuda_device, B, H, KV, hd, cap):
    """The fused decode-step op equals rope() on q|k heads, then kv_append(),
    then lens = pos + 1, bit for bit."""
    g = torch.Generator(device=cuda_device).manual_seed(B * H + hd)
    qkv = torch.randn((B, (H + 2 * KV) * hd), generator=g, device=cuda_device).half()
    pos = torch.randint(0, cap, (B,), generator=g, device=cuda_device, dtype=torch.int32)
    kc = torch.randn((B, KV, cap, hd), generator=g, device=cuda_device).half()
    vc = torch.randn_like(kc)
    q1, kc1, vc1 = qkv.clone(), kc.clone(), vc.clone()
    nb.rope(q1, H + KV, hd, positions=pos, theta=500000.0)
    nb.kv_append(q1[:, H * hd:(H + KV) * hd], q1[:, (H + KV) * hd:], kc1, vc1, pos=pos)
    lens = torch.full((B,), -7, dtype=torch.int32, device=cuda_device)
    nb.rope_kv_append(qkv, H, KV, hd, pos, kc, vc, theta=500000.0, lens=lens)
    assert torch.equal(qkv, q1)
    assert torch.equal(kc, kc1) and torch.equal(vc, vc1)
    assert torch.equal(lens, pos + 1)

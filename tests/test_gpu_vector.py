"""RMSNorm, SwiGLU, softmax and RoPE kernels against the oracle (GPU).
Tolerance: normwise relative error <= 1e-2 (TOL) unless stated."""
import numpy as np
import pytest
import torch

import npu_comp_b200 as nb
from oracle import ref

pytestmark = pytest.mark.gpu
TOL = 1e-2


def dev(a, d):
    return torch.from_numpy(np.ascontiguousarray(a)).to(d)


@pytest.mark.parametrize("rows,d", [(2048, 4096), (7, 64), (1, 8), (33, 11008)])
def test_rmsnorm(cuda_device, rng, rows, d):
    x = rng.standard_normal((rows, d)).astype(np.float16)
    g = (1 + 0.02 * rng.standard_normal(d)).astype(np.float16)
    y = nb.rmsnorm(dev(x, cuda_device), dev(g, cuda_device), 1e-5).float().cpu().numpy()
    assert ref.rel_err(y, ref.rmsnorm_ref(x, g, 1e-5)) <= TOL


def test_rmsnorm_fused_residual(cuda_device, rng):
    x = rng.standard_normal((64, 256)).astype(np.float16)
    r = rng.standard_normal((64, 256)).astype(np.float16)
    g = np.ones(256, np.float16)
    y, h = nb.rmsnorm(dev(x, cuda_device), dev(g, cuda_device), 1e-5, residual=dev(r, cuda_device))
    hs = (x.astype(np.float32) + r.astype(np.float32)).astype(np.float16)
    assert np.array_equal(h.cpu().numpy(), hs)  # fp16 round of an exact fp32 sum
    assert ref.rel_err(y.float().cpu().numpy(), ref.rmsnorm_ref(hs, g, 1e-5)) <= TOL


def test_rmsnorm_reference_example(cuda_device, examples):
    """The reference's RMSNorm example (test_rmsnorm.py, eps 0) within its own tolerance."""
    X, W = examples["rmsnorm_X"], examples["rmsnorm_W"]
    y = nb.rmsnorm(dev(X.astype(np.float16), cuda_device), dev(W.astype(np.float16), cuda_device), 0.0)
    got = y.float().cpu().numpy()
    assert np.abs(got - examples["rmsnorm_npu"]).max() < 1e-2  # test_rmsnorm.py:57
    assert np.abs(got - examples["rmsnorm_ref"]).max() < 1e-2


@pytest.mark.parametrize("rows,cols", [(2048, 11008), (3, 13), (8, 128)])
def test_swiglu(cuda_device, rng, rows, cols):
    gu = rng.standard_normal((rows, 2 * cols)).astype(np.float16)
    h = nb.swiglu(dev(gu, cuda_device)).float().cpu().numpy()
    assert ref.rel_err(h, ref.silu_mul_ref(gu[:, :cols], gu[:, cols:])) <= TOL


def test_swiglu_ffn_reference_example(cuda_device, examples):
    """The reference's SwiGLU FFN example (test_swiglu.py) built from our fp16 matmul and swiglu."""
    X, Wg, Wu, Wd = (examples[f"swiglu_{k}"].astype(np.float16) for k in ("X", "Wg", "Wu", "Wd"))
    x = dev(X, cuda_device)
    g = nb.matmul(x, dev(Wg.T, cuda_device))
    u = nb.matmul(x, dev(Wu.T, cuda_device))
    h = nb.swiglu(g, u)
    out = nb.matmul(h, dev(Wd.T, cuda_device)).float().cpu().numpy()
    assert ref.rel_err(out, examples["swiglu_npu"]) <= TOL
    assert ref.rel_err(out, examples["swiglu_ref"]) <= TOL


@pytest.mark.parametrize("causal,offset", [(False, 0), (True, 0), (True, 5)])
def test_softmax(cuda_device, rng, causal, offset):
    s = rng.standard_normal((3, 136, 256)).astype(np.float16)
    p = nb.softmax(dev(s, cuda_device), causal=causal, scale=0.7, causal_offset=offset).float().cpu().numpy()
    exp = ref.softmax_ref(s, 0.7, causal, offset)
    assert ref.rel_err(p, exp) <= TOL
    if causal:
        mask = np.arange(256)[None, :] > np.arange(136)[:, None] + offset
        assert np.all(p[:, mask] == 0.0)  # masked entries are exact zeros (exp(-30000) in the reference)


def test_softmax_prefill_shape(cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(3)
    s = torch.randn((32, 2048, 2048), generator=g, device=cuda_device).half()
    p = nb.softmax(s, causal=True)
    sub = s[5, 1000:1010].float().cpu().numpy()
    ref_rows = ref.softmax_ref(sub, 1.0, True, offset=1000)
    assert ref.rel_err(p[5, 1000:1010].float().cpu().numpy(), ref_rows) <= TOL
    rows = p.float().sum(-1)
    assert torch.allclose(rows, torch.ones_like(rows), atol=2e-2)


@pytest.mark.parametrize("T,H,hd,pos0", [(64, 4, 128, 0), (8, 4, 16, 3), (5, 2, 64, 4096)])
def test_rope(cuda_device, rng, T, H, hd, pos0):
    x = rng.standard_normal((T, H * hd + 16)).astype(np.float16)
    xt = dev(x, cuda_device)
    nb.rope(xt, H, hd, pos0=pos0)
    got = xt.float().cpu().numpy()
    exp = ref.rope_ref(x[:, :H * hd], H, hd, np.arange(T) + pos0)
    assert ref.rel_err(got[:, :H * hd], exp) <= TOL
    assert np.array_equal(got[:, H * hd:], x[:, H * hd:].astype(np.float32))  # columns past the heads untouched


def test_rope_positions_tensor(cuda_device, rng):
    T, H, hd = 6, 2, 32
    pos = np.array([0, 7, 3, 4095, 1, 2], np.int32)
    x = rng.standard_normal((T, H * hd)).astype(np.float16)
    xt = dev(x, cuda_device)
    nb.rope(xt, H, hd, positions=dev(pos, cuda_device))
    assert ref.rel_err(xt.float().cpu().numpy(), ref.rope_ref(x, H, hd, pos)) <= TOL


@pytest.mark.parametrize("rows,cols", [(64, 4096), (33, 1000)])
def test_residual_add(cuda_device, rng, rows, cols):
    a = rng.standard_normal((rows, cols)).astype(np.float16)
    b = rng.standard_normal((rows, cols)).astype(np.float16)
    got = nb.add(dev(a, cuda_device), dev(b, cuda_device)).cpu().numpy()
    assert np.array_equal(got, (a.astype(np.float32) + b.astype(np.float32)).astype(np.float16))  # exact


@pytest.mark.parametrize("ranks", [1, 2, 4, 8])
def test_greedy_keys_select_the_global_argmax(cuda_device, rng, ranks):
    """argmax_keys on each vocabulary shard + select_keys over the gathered keys
    == the argmax of the whole row (largest value, smallest index on ties),
    including ties placed across shards and all-negative rows."""
    B, V = 9, 4096
    x = rng.standard_normal((B, V)).astype(np.float16)
    x[1, 100] = x[1, 3000] = 7.0        # tie across shards: the smaller index wins
    x[2, 5] = x[2, 6] = 9.0             # tie inside a shard
    x[3] = -np.abs(x[3]) - 1.0          # no positive logit
    x[4, V - 1] = 11.0                  # the last index
    xt = dev(x, cuda_device)
    vs = V // ranks
    keys = torch.cat([nb.npu.argmax_keys(xt[:, r * vs:(r + 1) * vs].contiguous(), r * vs) for r in range(ranks)])
    ids = nb.npu.select_keys(keys, ranks).cpu().numpy()
    assert np.array_equal(ids, np.argmax(x.astype(np.float32), axis=1))
    idx, _ = nb.argmax(xt)
    assert np.array_equal(idx.cpu().numpy(), ids)


@pytest.mark.parametrize("rows,cols,ld", [(32, 32000, 32000), (5, 32003, 32003), (3, 1001, 1005), (2, 7, 7)])
def test_argmax_rows_vector_and_scalar_paths(cuda_device, rng, rows, cols, ld):
    """The per-row argmax against numpy's (first index on ties): 16-byte loads
    where a row starts 16-byte aligned, scalar elsewhere and for the tail;
    ties inside one vector, across vectors and at the last column."""
    x = rng.standard_normal((rows, ld)).astype(np.float16)
    x[0, 3] = x[0, 5] = 12.0                     # tie inside a vector
    if cols > 20:
        x[1 % rows, 9] = x[1 % rows, cols - 1] = 13.0   # tie across vectors / the tail
    x[rows - 1, cols - 1] = 20.0                 # the last column
    xt = dev(x, cuda_device)[:, :cols]
    idx, val = nb.argmax(xt)
    want = np.argmax(x[:, :cols].astype(np.float32), axis=1)
    assert np.array_equal(idx.cpu().numpy(), want)
    assert np.array_equal(val.cpu().numpy(), x[np.arange(rows), want].astype(np.float32))

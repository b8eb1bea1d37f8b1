"""The oracle's float64 layer over quantised, fused weights (ref_layer_q,
ref_decode_layer_q, ref_stack_logits) against ref_layer, which
test_oracle_goldens pins to the reference's own float layer
(d_compiler/npu_compiler/model.py:115-157 via llama_layer.py's output).

The GPU tests at the benchmarked sizes compare with these functions, so they
must agree with ref_layer to float64 rounding on the reference's own layer and
on a GQA layer with random weights."""
import numpy as np
import pytest

from oracle import ref
from tests.test_gpu_layer import layer_weights_from_fixture


def fused(W, H, KV, F):
    """The build's layout of the reference weight dict: fused, quantised,
    gate|up rows interleaved."""
    names = [f"Wq{h}" for h in range(H)] + [f"Wk{k}" for k in range(KV)] + [f"Wv{k}" for k in range(KV)]
    wqkv, sqkv = ref.quantize_w8(np.concatenate([np.asarray(W[n], np.float32) for n in names], 1))
    wo, so = ref.quantize_w8(np.concatenate([np.asarray(W[f"Wo{h}"], np.float32) for h in range(H)], 0))
    gu, sgu = ref.quantize_w8(np.concatenate([np.asarray(W["Wg"], np.float32), np.asarray(W["Wu"], np.float32)], 1))
    wgu, sg = np.empty_like(gu), np.empty_like(sgu)
    wgu[0::2], wgu[1::2] = gu[:F], gu[F:]
    sg[0::2], sg[1::2] = sgu[:F], sgu[F:]
    wd, sd = ref.quantize_w8(np.asarray(W["Wd"], np.float32))
    return dict(wqkv=wqkv, sqkv=sqkv, wo=wo, so=so, wgu=wgu, sgu=sg, wd=wd, sd=sd, g1=W["Wn1"], g2=W["Wn2"])


def random_layer(rng, D, H, KV, HD, F):
    W = {"Wn1": rng.uniform(0.8, 1.2, D), "Wn2": rng.uniform(0.8, 1.2, D), "Wg": rng.uniform(-.2, .2, (D, F)),
         "Wu": rng.uniform(-.2, .2, (D, F)), "Wd": rng.uniform(-.2, .2, (F, D))}
    for h in range(H):
        W[f"Wq{h}"] = rng.uniform(-.2, .2, (D, HD))
        W[f"Wo{h}"] = rng.uniform(-.2, .2, (HD, D))
    for k in range(KV):
        W[f"Wk{k}"] = rng.uniform(-.2, .2, (D, HD))
        W[f"Wv{k}"] = rng.uniform(-.2, .2, (D, HD))
    return {k: v.astype(np.float32) for k, v in W.items()}


def test_fused_layer_equals_ref_layer_on_the_reference_layer(examples):
    W, (SEQ, D, H, KV, HD, F) = layer_weights_from_fixture(examples)
    cos, sin = ref.rope_tables(SEQ, HD)
    want = ref.ref_layer(ref.quantized_weights(W, H, KV), examples["layer_X"], H, KV, HD, 0.0, cos, sin)
    got = ref.ref_layer_q(fused(W, H, KV, F), examples["layer_X"], H, KV, HD, 0.0)
    assert np.abs(got - want).max() <= 1e-12 * np.abs(want).max()


@pytest.mark.parametrize("H,KV", [(4, 2), (4, 4), (8, 2)])
def test_fused_layer_and_decode_step_equal_ref_layer(rng, H, KV):
    D, HD, F, T = 64, 16, 96, 11
    W = random_layer(rng, D, H, KV, HD, F)
    L = fused(W, H, KV, F)
    x = rng.standard_normal((T, D))
    cos, sin = ref.rope_tables(T, HD)
    want = ref.ref_layer(ref.quantized_weights(W, H, KV), x, H, KV, HD, 1e-5, cos, sin)
    got = ref.ref_layer_q(L, x, H, KV, HD, 1e-5)
    assert np.abs(got - want).max() <= 1e-12 * np.abs(want).max()
    # decode: the cached (rotated) keys and values of positions < T - 1, then row T - 1
    P = ref.prepare_layer(L)
    qkv = ref._rms64(x, P["g1"], 1e-5) @ P["qkv"].T
    k = ref._rope64(qkv[:, H * HD:(H + KV) * HD], KV, HD, np.arange(T), 1e4)
    v = qkv[:, (H + KV) * HD:]
    kc = k.reshape(T, KV, HD).transpose(1, 0, 2)[None]
    vc = v.reshape(T, KV, HD).transpose(1, 0, 2)[None]
    yd = ref.ref_decode_layer_q(L, x[T - 1:], kc, vc, np.array([T - 1]), H, KV, HD, 1e-5)
    assert np.abs(yd[0] - want[T - 1]).max() <= 1e-12 * np.abs(want).max()


def test_stack_logits_compose_layers(rng):
    D, H, KV, HD, F, V, T = 64, 4, 2, 16, 96, 50, 7
    Ls = [fused(random_layer(rng, D, H, KV, HD, F), H, KV, F) for _ in range(2)]
    emb = rng.standard_normal((V, D)).astype(np.float16)
    lm = (rng.standard_normal((V, D)) * 0.05).astype(np.float16)
    norm = np.ones(D, np.float16)
    toks = rng.integers(0, V, (2, T))
    got = ref.ref_stack_logits(iter(Ls), emb, norm, lm, toks, H, KV, HD, 1e-5, rows=np.array([T - 2, T - 1]))
    for b in range(2):
        x = emb[toks[b]].astype(np.float64)
        for L in Ls:
            x = ref.ref_layer_q(L, x, H, KV, HD, 1e-5)
        want = ref._rms64(x, norm, 1e-5) @ lm.astype(np.float64).T
        assert np.allclose(got[b], want[T - 2:], rtol=0, atol=1e-12)
        # causality: the logits of row T - 2 do not depend on the last token
        t2 = toks[b].copy()
        t2[-1] = (t2[-1] + 1) % V
        x2 = emb[t2].astype(np.float64)
        for L in Ls:
            x2 = ref.ref_layer_q(L, x2, H, KV, HD, 1e-5)
        assert np.allclose((ref._rms64(x2, norm, 1e-5) @ lm.astype(np.float64).T)[T - 2], want[T - 2], atol=1e-12)

"""numpy references for the hot path -- TEST INFRASTRUCTURE ONLY (the checker).

Each function restates a reference computation, citing the file it follows
(paths inside KwanyoungCho/NPU_COMP):
  * per-save fp16 references of the example scripts
    (b_program_examples/test_matmul.py:22, test_rmsnorm.py:45-48,
    test_swiglu.py:41-46, test_attention.py:57-69);
  * tiled_fp16_ref  (d_compiler/tests/test_tiling.py:37-47);
  * float64 ref_layer  (d_compiler/npu_compiler/model.py:115-157) and the RoPE
    tables with the Llama-3 frequency scaling
    (d_compiler/npu_compiler/legalize.py:50-85);
  * the W8A16 quantisation, which the reference does not have: symmetric per
    output channel, scale = fp16(absmax / 127), q = clip(rint(W / scale), +-127).
    Parity of that part is unpinned by any reference test; it is pinned here by
    known-answer cases (power-of-two scales, +-127 extremes, K = 1).
"""
from __future__ import annotations

import math
from typing import Dict, Optional

import numpy as np


def f16(x) -> np.ndarray:
    """Round through fp16 (RNE) and back to float32 -- the cmodel's save, or
    npu.fp16() of a python double (float64 input is rounded directly, with no
    intermediate float32 rounding)."""
    x = np.asarray(x)
    if x.dtype != np.float64:
        x = x.astype(np.float32)
    return x.astype(np.float16).astype(np.float32)


# ------------------------------------------------------------------ W8A16

def quantize_w8(W: np.ndarray):
    """W [K, N] float32 -> (q int8 [N, K], s fp16 [N])."""
    W = np.asarray(W, dtype=np.float32)
    amax = np.abs(W).max(axis=0)
    s = (amax / np.float32(127.0)).astype(np.float16)
    sf = s.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(sf[None, :] > 0, np.rint(W / np.where(sf > 0, sf, 1)[None, :]), 0)
    q = np.clip(q, -127, 127).astype(np.int8)
    return np.ascontiguousarray(q.T), s


def dequant_f16(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    """fp16(q * s) as the NPU's fp16 weight matrix, laid out [K, N] (x @ W)."""
    return f16(q.astype(np.float32) * s.astype(np.float32)[:, None]).T.copy()


def w8a16_ref(A: np.ndarray, q: np.ndarray, s: np.ndarray, residual: Optional[np.ndarray] = None,
              alpha: float = 1.0) -> np.ndarray:
    """Exact float64 value of the build's W8A16 matmul before its fp16 store:
    alpha * s[n] * sum_k A[m,k] q[n,k] (+ residual)."""
    acc = A.astype(np.float64) @ q.astype(np.float64).T
    out = alpha * acc * s.astype(np.float64)[None, :]
    if residual is not None:
        out = out + residual.astype(np.float64)
    return out


def matmul_f16_ref(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """One-shot NPU matmul: fp16(sum_k f32 A * f32 B) (mysim.cpp:109-113)."""
    return f16(A.astype(np.float32) @ B.astype(np.float32))


def matmul_f16_pyref(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """The example scripts' reference matmul: fp16 of a double-precision sum
    (test_matmul.py:22, test_swiglu.py:40, test_attention.py:58)."""
    return f16(A.astype(np.float64) @ B.astype(np.float64))


def tiled_fp16_ref(A: np.ndarray, B: np.ndarray, T: int = 64) -> np.ndarray:
    """64-tiled NPU matmul: C = fp16(C + fp16(A_k @ B_k)) (test_tiling.py:37-47)."""
    A = A.astype(np.float32)
    B = B.astype(np.float32)
    C = None
    for kk in range(0, A.shape[1], T):
        part = f16(A[:, kk:kk + T] @ B[kk:kk + T, :])
        C = part if C is None else f16(C + part)
    return C


def rel_err(got, ref) -> float:
    """Normwise relative error max|got - ref| / max|ref| (the reference's
    convention, d_compiler/tests/test_matmul.py:47-48, llama_layer.py:199-202)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.abs(ref).max()
    return float(np.abs(got - ref).max() / (den if den > 0 else 1.0))


# ------------------------------------------------------------- vector ops

def rmsnorm_ref(x: np.ndarray, g: np.ndarray, eps: float) -> np.ndarray:
    """model.py:121-123: x / sqrt(mean(x^2) + eps) * w, float64."""
    x = x.astype(np.float64)
    ms = np.mean(x * x, axis=-1, keepdims=True) + eps
    return x / np.sqrt(ms) * g.astype(np.float64)


def rmsnorm_npu_ref(X: np.ndarray, W: np.ndarray) -> np.ndarray:
    """Per-save fp16 RMSNorm of test_rmsnorm.py:45-48 (eps 0): the sum of
    squares and 1/sqrt in double, then fp16(fp16(x * fp16(inv)) * w)."""
    X = np.asarray(X, dtype=np.float64)
    out = np.empty_like(X, dtype=np.float32)
    D = X.shape[1]
    for i in range(X.shape[0]):
        ms = float(np.sum(X[i] * X[i])) / D
        inv = f16(1.0 / math.sqrt(ms))
        out[i] = f16(f16(f16(X[i].astype(np.float32) * inv)) * W.astype(np.float32))
    return out


def silu_mul_ref(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """legalize.py:130-149: g / (1 + exp(-g)) * u, float64."""
    g = g.astype(np.float64)
    return g / (1.0 + np.exp(-g)) * u.astype(np.float64)


def swiglu_npu_ref(G: np.ndarray, U: np.ndarray) -> np.ndarray:
    """Per-save fp16 SiLU*up of test_swiglu.py:43-46 (python doubles between saves)."""
    G = G.astype(np.float64)
    with np.errstate(over="ignore"):
        sig = f16(1.0 / f16(1.0 + f16(np.exp(-G))).astype(np.float64)).astype(np.float64)
    silu = f16(G * sig).astype(np.float64)
    return f16(silu * U.astype(np.float64))


def softmax_ref(s: np.ndarray, scale: float = 1.0, causal: bool = False, offset: int = 0) -> np.ndarray:
    """Stable row softmax of scale*s (model.py:145-150); causal rows r see c <= r + offset."""
    x = s.astype(np.float64) * scale
    if causal:
        R, C = x.shape[-2], x.shape[-1]
        mask = np.arange(C)[None, :] > (np.arange(R)[:, None] + offset)
        x = np.where(mask, -np.inf, x)
    x = x - x.max(axis=-1, keepdims=True)
    e = np.exp(x)
    return e / e.sum(axis=-1, keepdims=True)


def llama3_scale_freqs(freqs: np.ndarray, factor: float = 32.0, low: float = 1.0, high: float = 4.0,
                       old_ctx: float = 8192.0) -> np.ndarray:
    """Llama-3 RoPE frequency scaling of legalize.py:50-64, float64: frequencies
    whose wavelength exceeds old_ctx/low are divided by factor, those below
    old_ctx/high kept, the band between blended linearly in old_ctx/wavelength."""
    out = np.empty_like(np.asarray(freqs, dtype=np.float64))
    for i, f in enumerate(np.asarray(freqs, dtype=np.float64)):
        wl = 2.0 * np.pi / f
        if wl > old_ctx / low:
            out[i] = f / factor
        elif wl < old_ctx / high:
            out[i] = f
        else:
            sm = (old_ctx / wl - low) / (high - low)
            out[i] = (1.0 - sm) * f / factor + sm * f
    return out


def rope_freqs(hd: int, base: float = 10000.0, llama3_scaling=False) -> np.ndarray:
    """base^(-2i/hd) for i < hd/2 (legalize.py:71), Llama-3 scaled when
    llama3_scaling is True (the reference's constants) or a tuple (factor,
    low, high, old_ctx) (legalize.py:72-73)."""
    freqs = base ** (-2.0 * np.arange(hd // 2) / hd)
    if llama3_scaling is True:
        freqs = llama3_scale_freqs(freqs)
    elif llama3_scaling:
        freqs = llama3_scale_freqs(freqs, *llama3_scaling)
    return freqs


def rope_tables(seq: int, hd: int, base: float = 10000.0, pos0: int = 0, llama3_scaling=False):
    """Host cos/sin tables of legalize.py:67-85, [seq, hd] (float64)."""
    freqs = rope_freqs(hd, base, llama3_scaling)
    ang = (np.arange(seq)[:, None] + pos0) * freqs[None, :]
    cos = np.concatenate([np.cos(ang), np.cos(ang)], axis=1)
    sin = np.concatenate([np.sin(ang), np.sin(ang)], axis=1)
    return cos, sin


def rope_ref(x: np.ndarray, heads: int, hd: int, positions: np.ndarray, theta: float = 10000.0) -> np.ndarray:
    """x' = x*cos + rotate_half(x)*sin per head (llama_layer.py:96-112, model.py:125-131), float64."""
    x = x.astype(np.float64).copy()
    T = x.shape[0]
    half = hd // 2
    freqs = theta ** (-2.0 * np.arange(half) / hd)
    ang = positions.astype(np.float64)[:, None] * freqs[None, :]
    c, s = np.cos(ang), np.sin(ang)
    for h in range(heads):
        a = x[:, h * hd: h * hd + half].copy()
        b = x[:, h * hd + half: (h + 1) * hd].copy()
        x[:, h * hd: h * hd + half] = a * c - b * s
        x[:, h * hd + half: (h + 1) * hd] = b * c + a * s
    return x[:, : heads * hd] if x.shape[1] > heads * hd else x


def attention_ref(q, k, v, heads: int, kv_heads: int, hd: int, causal: bool = True,
                  scale: Optional[float] = None) -> np.ndarray:
    """GQA attention of llama_layer.py:114-137 / model.py:140-152 in float64 for
    one sequence: q [T, heads*hd], k/v [T, kv_heads*hd] -> [T, heads*hd]."""
    scale = 1.0 / math.sqrt(hd) if scale is None else scale
    T = q.shape[0]
    out = np.zeros((T, heads * hd))
    grp = heads // kv_heads
    for h in range(heads):
        kv = h // grp
        Q = q[:, h * hd:(h + 1) * hd].astype(np.float64)
        K = k[:, kv * hd:(kv + 1) * hd].astype(np.float64)
        V = v[:, kv * hd:(kv + 1) * hd].astype(np.float64)
        P = softmax_ref(Q @ K.T, scale, causal)
        out[:, h * hd:(h + 1) * hd] = P @ V
    return out


def decode_attention_ref(q, kc, vc, lens, heads, kv_heads, hd, scale=None) -> np.ndarray:
    """One query per sequence against caches [B, KVH, cap, hd], float64."""
    scale = 1.0 / math.sqrt(hd) if scale is None else scale
    B = q.shape[0]
    grp = heads // kv_heads
    out = np.zeros((B, heads * hd))
    for b in range(B):
        L = int(lens[b])
        for h in range(heads):
            kv = h // grp
            Q = q[b, h * hd:(h + 1) * hd].astype(np.float64)
            K = kc[b, kv, :L].astype(np.float64)
            V = vc[b, kv, :L].astype(np.float64)
            s = (K @ Q) * scale
            p = np.exp(s - s.max())
            out[b, h * hd:(h + 1) * hd] = (p / p.sum()) @ V
    return out


# ---------------------------------------------------------------- layer

def ref_layer(W: Dict[str, np.ndarray], x: np.ndarray, H: int, KV: int, HD: int, eps: float,
              cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """float64 Llama layer of model.py:115-157 (GQA, rotate_half RoPE from
    host tables, causal softmax, SwiGLU FFN, two residuals).  Weights in the
    reference's layout: Wq{h}/Wk{k}/Wv{k} [D, HD], Wo{h} [HD, D], Wg/Wu [D, F],
    Wd [F, D], Wn1/Wn2 [D]."""
    SEQ = x.shape[0]
    GPK = H // KV
    half = HD // 2
    x = x.astype(np.float64)

    def rms(X, w):
        ms = np.mean(X ** 2, axis=1, keepdims=True) + eps
        return X / np.sqrt(ms) * np.asarray(w, dtype=np.float64).reshape(1, -1)

    def rope_apply(M):
        rh = np.concatenate([-M[:, half:], M[:, :half]], axis=1)
        return M * cos[:SEQ] + rh * sin[:SEQ]

    f = lambda n: np.asarray(W[n], dtype=np.float64)  # noqa: E731
    Xn = rms(x, W["Wn1"])
    Kt, Vh = {}, {}
    for k in range(KV):
        Kt[k] = rope_apply(Xn @ f(f"Wk{k}")).T
        Vh[k] = Xn @ f(f"Wv{k}")
    attn = np.zeros((SEQ, x.shape[1]))
    mask = np.triu(np.ones((SEQ, SEQ), dtype=bool), 1)
    for h in range(H):
        kv = h // GPK
        Q = rope_apply(Xn @ f(f"Wq{h}"))
        S = (Q @ Kt[kv]) / np.sqrt(HD)
        S[mask] = -np.inf
        S = S - S.max(axis=1, keepdims=True)
        e = np.exp(S)
        P = e / e.sum(axis=1, keepdims=True)
        attn += (P @ Vh[kv]) @ f(f"Wo{h}")
    hres = x + attn
    Hn = rms(hres, W["Wn2"])
    gate = Hn @ f("Wg")
    up = Hn @ f("Wu")
    ffn = (gate / (1.0 + np.exp(-gate)) * up) @ f("Wd")
    return hres + ffn


def quantized_weights(W: Dict[str, np.ndarray], H: int, KV: int) -> Dict[str, np.ndarray]:
    """The float weights a W8A16 layer actually applies: every linear replaced by
    its per-output-channel dequantisation q*s (exact, float64), quantised over
    the fused matrices the build uses (QKV, O, gate|up, down)."""
    out = dict(W)
    D = np.asarray(W["Wn1"]).size
    HD = np.asarray(W["Wq0"]).shape[1]
    names = [f"Wq{h}" for h in range(H)] + [f"Wk{k}" for k in range(KV)] + [f"Wv{k}" for k in range(KV)]
    qkv = np.concatenate([np.asarray(W[n], dtype=np.float32) for n in names], axis=1)
    q, s = quantize_w8(qkv)
    dq = (q.astype(np.float64) * s.astype(np.float64)[:, None]).T
    for i, n in enumerate(names):
        out[n] = dq[:, i * HD:(i + 1) * HD]
    wo = np.concatenate([np.asarray(W[f"Wo{h}"], dtype=np.float32) for h in range(H)], axis=0)
    q, s = quantize_w8(wo)
    dq = (q.astype(np.float64) * s.astype(np.float64)[:, None]).T
    for h in range(H):
        out[f"Wo{h}"] = dq[h * HD:(h + 1) * HD]
    F = np.asarray(W["Wg"]).shape[1]
    gu = np.concatenate([np.asarray(W["Wg"], dtype=np.float32), np.asarray(W["Wu"], dtype=np.float32)], axis=1)
    q, s = quantize_w8(gu)
    dq = (q.astype(np.float64) * s.astype(np.float64)[:, None]).T
    out["Wg"], out["Wu"] = dq[:, :F], dq[:, F:]
    q, s = quantize_w8(np.asarray(W["Wd"], dtype=np.float32))
    out["Wd"] = (q.astype(np.float64) * s.astype(np.float64)[:, None]).T
    assert out["Wd"].shape == (F, D)
    return out


# ------------------------------------------ layer on quantised, fused weights
#
# The same float64 layer as ref_layer (model.py:115-157), written over the
# weights in the layout the W8A16 build stores them: int8 q [N, K] with fp16
# per-output-channel scales s [N] (applied exactly: q * s in float64), QKV
# fused as [q heads | k heads | v heads] rows, gate|up rows interleaved
# (row 2c gate channel c, row 2c + 1 up channel c).  Used at full Llama-7B
# size, where the per-head weight dict of ref_layer is not at hand.

def dequant(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    """float64 q[n, k] * s[n] (exact: an 8-bit integer times an fp16 value)."""
    out = q.astype(np.float64)
    np.multiply(out, s.astype(np.float64)[:, None], out=out)
    return out


def _rms64(X: np.ndarray, g: np.ndarray, eps: float) -> np.ndarray:
    ms = np.mean(X * X, axis=1, keepdims=True) + eps
    return X / np.sqrt(ms) * np.asarray(g, dtype=np.float64).reshape(1, -1)


def _rope64(M: np.ndarray, heads: int, hd: int, positions: np.ndarray, theta: float,
            inv_freq: Optional[np.ndarray] = None) -> np.ndarray:
    """rotate_half RoPE (model.py:125-131) of every head of M [T, heads*hd] at
    the given positions; inv_freq [hd/2] overrides theta^(-2i/hd)."""
    half = hd // 2
    freqs = theta ** (-2.0 * np.arange(half) / hd) if inv_freq is None else np.asarray(inv_freq, np.float64)
    ang = positions.astype(np.float64)[:, None] * freqs[None, :]
    c, s = np.cos(ang), np.sin(ang)
    X = M.reshape(M.shape[0], heads, hd)
    a, b = X[:, :, :half], X[:, :, half:]
    out = np.concatenate([a * c[:, None, :] - b * s[:, None, :], b * c[:, None, :] + a * s[:, None, :]], axis=2)
    return out.reshape(M.shape[0], heads * hd)


def prepare_layer(L: Dict[str, np.ndarray]) -> Dict[str, np.ndarray]:
    """The float64 matrices a quantised layer applies ([N, K] each), computed
    once; ref_layer_q and ref_decode_layer_q accept either form."""
    if "qkv" in L:
        return L
    return {"qkv": dequant(L["wqkv"], L["sqkv"]), "o": dequant(L["wo"], L["so"]),
            "gu": dequant(L["wgu"], L["sgu"]), "d": dequant(L["wd"], L["sd"]),
            "g1": np.asarray(L["g1"], np.float64), "g2": np.asarray(L["g2"], np.float64)}


def ref_layer_q(L: Dict[str, np.ndarray], x: np.ndarray, heads: int, kv_heads: int, hd: int, eps: float,
                theta: float = 10000.0, positions: Optional[np.ndarray] = None,
                inv_freq: Optional[np.ndarray] = None) -> np.ndarray:
    """float64 causal Llama layer for one sequence x [T, d] on quantised weights
    L = {wqkv, sqkv, wo, so, wgu, sgu, wd, sd, g1, g2} (module comment above),
    or on prepare_layer(L)."""
    P = prepare_layer(L)
    T = x.shape[0]
    pos = np.arange(T) if positions is None else np.asarray(positions)
    x = x.astype(np.float64)
    qd, kd = heads * hd, kv_heads * hd
    xn = _rms64(x, P["g1"], eps)
    qkv = xn @ P["qkv"].T
    q = _rope64(qkv[:, :qd], heads, hd, pos, theta, inv_freq)
    k = _rope64(qkv[:, qd:qd + kd], kv_heads, hd, pos, theta, inv_freq)
    v = qkv[:, qd + kd:qd + 2 * kd]
    ctx = np.zeros((T, qd))
    grp = heads // kv_heads
    mask = np.triu(np.ones((T, T), dtype=bool), 1)
    for h in range(heads):
        kv = h // grp
        S = (q[:, h * hd:(h + 1) * hd] @ k[:, kv * hd:(kv + 1) * hd].T) / math.sqrt(hd)
        S[mask] = -np.inf
        S -= S.max(axis=1, keepdims=True)
        E = np.exp(S)
        E /= E.sum(axis=1, keepdims=True)
        ctx[:, h * hd:(h + 1) * hd] = E @ v[:, kv * hd:(kv + 1) * hd]
    h_ = x + ctx @ P["o"].T
    return h_ + _ffn64(P, _rms64(h_, P["g2"], eps))


def _ffn64(P: Dict[str, np.ndarray], hn: np.ndarray) -> np.ndarray:
    gu = hn @ P["gu"].T
    g, u = gu[:, 0::2], gu[:, 1::2]
    return (g / (1.0 + np.exp(-g)) * u) @ P["d"].T


def ref_decode_layer_q(L: Dict[str, np.ndarray], x: np.ndarray, k_cache, v_cache, pos: np.ndarray, heads: int,
                       kv_heads: int, hd: int, eps: float, theta: float = 10000.0,
                       inv_freq: Optional[np.ndarray] = None) -> np.ndarray:
    """One decode step of the float64 layer: x [B, d] is the token at position
    pos[b] of sequence b; k_cache / v_cache [B, kv_heads, >= pos[b], hd] hold
    the (already rotated) keys and the values of positions 0 .. pos[b] - 1.
    The token's own k and v join them; attention covers pos[b] + 1 keys."""
    P = prepare_layer(L)
    B = x.shape[0]
    x = x.astype(np.float64)
    qd, kd = heads * hd, kv_heads * hd
    xn = _rms64(x, P["g1"], eps)
    qkv = xn @ P["qkv"].T
    pos = np.asarray(pos)
    q = _rope64(qkv[:, :qd], heads, hd, pos, theta, inv_freq)
    k = _rope64(qkv[:, qd:qd + kd], kv_heads, hd, pos, theta, inv_freq)
    v = qkv[:, qd + kd:qd + 2 * kd]
    grp = heads // kv_heads
    ctx = np.zeros((B, qd))
    for b in range(B):
        n = int(pos[b])
        Kb = np.concatenate([np.asarray(k_cache[b, :, :n], dtype=np.float64),
                             k[b].reshape(kv_heads, 1, hd)], axis=1)          # [KV, n + 1, hd]
        Vb = np.concatenate([np.asarray(v_cache[b, :, :n], dtype=np.float64),
                             v[b].reshape(kv_heads, 1, hd)], axis=1)
        Q = q[b].reshape(kv_heads, grp, hd)
        S = np.einsum("kgd,ktd->kgt", Q, Kb) / math.sqrt(hd)
        S -= S.max(axis=2, keepdims=True)
        E = np.exp(S)
        E /= E.sum(axis=2, keepdims=True)
        ctx[b] = np.einsum("kgt,ktd->kgd", E, Vb).reshape(qd)
    h_ = x + ctx @ P["o"].T
    return h_ + _ffn64(P, _rms64(h_, P["g2"], eps))


def ref_stack_logits(layers, embed: np.ndarray, norm: np.ndarray, lm_head: np.ndarray, tokens: np.ndarray,
                     heads: int, kv_heads: int, hd: int, eps: float, theta: float = 10000.0,
                     rows: Optional[np.ndarray] = None, inv_freq: Optional[np.ndarray] = None) -> np.ndarray:
    """float64 decoder stack on sequences of token ids tokens [B, T]: embedding
    rows (fp16 table), the layers (an iterable of ref_layer_q weight dicts,
    each prepared once and applied to every sequence), final RMSNorm and the
    lm_head [vocab, d] -> logits [B, len(rows), vocab] of `rows` (default:
    every position).  Greedy decoding feeds the chosen tokens back as later
    positions, so the logits of decode step s are row T - 1 + s of one pass
    over the prompt followed by the generated tokens."""
    from concurrent.futures import ThreadPoolExecutor
    tokens = np.atleast_2d(np.asarray(tokens))
    emb = np.asarray(embed)
    xs = [emb[t].astype(np.float64) for t in tokens]
    it = iter(layers)
    with ThreadPoolExecutor(max_workers=4) as ex:  # dequantise the next layers while one is applied
        while True:
            group = [L for _, L in zip(range(4), it)]
            if not group:
                break
            for P in ex.map(prepare_layer, group):
                xs = [ref_layer_q(P, x, heads, kv_heads, hd, eps, theta, inv_freq=inv_freq) for x in xs]
    rows = np.arange(tokens.shape[1]) if rows is None else np.asarray(rows)
    lm = np.asarray(lm_head, dtype=np.float64)
    return np.stack([_rms64(x[rows], norm, eps) @ lm.T for x in xs])

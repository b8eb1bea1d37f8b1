"""W8A16 matmul on the GPU (tcgen05 2-CTA pairs) against the oracle.

Tolerance (floating point, fp16 output): normwise relative error
max|got - ref| / max|ref| <= 1e-2 (TOL); integer quantisation is bit-exact.
"""
import os

import numpy as np
import pytest
import torch

import npu_comp_b200 as nb
from oracle import ref

pytestmark = pytest.mark.gpu
TOL = 1e-2
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def to_dev(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def test_config1_against_reference_simulator(cuda_device):
    """The single W8A16 matmul configuration vs the reference's CPU path (mysim
    running the compiler's 64-tiled program on dequantised weights)."""
    rng = np.random.default_rng(0)
    A = rng.standard_normal((64, 512)).astype(np.float16)
    W = (rng.standard_normal((512, 512)) * 0.02).astype(np.float32)
    q, s = ref.quantize_w8(W)
    qd, sd = nb.quantize_w8(to_dev(W, cuda_device))
    assert np.array_equal(qd.cpu().numpy(), q) and np.array_equal(sd.cpu().numpy(), s)
    C = nb.matmul(to_dev(A, cuda_device), qd, sd).float().cpu().numpy()
    C_mysim = np.load(os.path.join(GOLDEN, "w8a16_config1.npz"))["C_mysim"].astype(np.float32)
    exact = ref.w8a16_ref(A, q, s)
    assert ref.rel_err(C, C_mysim) <= TOL
    assert ref.rel_err(C, exact) <= TOL
    # the GPU keeps fp32 accumulation to the end: closer to exact than the fp16 tiled program
    assert ref.rel_err(C, exact) <= ref.rel_err(C_mysim, exact)
    assert np.abs(C - exact).mean() < 2e-3


@pytest.mark.parametrize("K,N", [(512, 512), (4096, 300), (1, 33), (64, 7)])
def test_quantizer_bit_exact(cuda_device, rng, K, N):
    W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    W[:, 0] = 0.0  # a zero column
    q, s = ref.quantize_w8(W)
    qd, sd = nb.quantize_w8(to_dev(W, cuda_device))
    assert np.array_equal(qd.cpu().numpy(), q)
    assert np.array_equal(sd.cpu().numpy().view(np.uint16), s.view(np.uint16))


SHAPES = [(64, 512, 512), (1, 1000, 256), (8, 64, 64), (128, 128, 64), (200, 300, 160), (129, 257, 96),
          (333, 777, 1024), (64, 12288, 4096), (64, 4096, 1376), (512, 256, 11008), (2048, 4096, 4096),
          (32, 22016, 4096), (48, 1000, 4096), (16, 11008, 512), (64, 4096, 11008), (3, 128, 16),
          (400, 300, 160), (1000, 777, 1376), (385, 257, 96), (4096, 512, 4096)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_w8a16_shapes(cuda_device, rng, M, N, K):
    A = rng.standard_normal((M, K)).astype(np.float16)
    W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    q, s = ref.quantize_w8(W)
    C = nb.matmul(to_dev(A, cuda_device), to_dev(q, cuda_device), to_dev(s, cuda_device)).float().cpu().numpy()
    assert C.shape == (M, N)
    assert ref.rel_err(C, ref.w8a16_ref(A, q, s)) <= TOL


def test_w8a16_residual_alpha_and_strided_output(cuda_device, rng):
    M, N, K = 300, 500, 128
    A = rng.standard_normal((M, K)).astype(np.float16)
    q = rng.integers(-127, 128, (N, K)).astype(np.int8)
    s = (rng.uniform(0.5, 2, N) * 1e-3).astype(np.float16)
    R = rng.standard_normal((M, N)).astype(np.float16)
    out = torch.zeros((M, N + 24), dtype=torch.float16, device=cuda_device)[:, 8:8 + N]
    nb.matmul(to_dev(A, cuda_device), to_dev(q, cuda_device), to_dev(s, cuda_device), out=out,
              residual=to_dev(R, cuda_device), alpha=0.5)
    got = out.float().cpu().numpy()
    assert ref.rel_err(got, ref.w8a16_ref(A, q, s, residual=R, alpha=0.5)) <= TOL


def test_w8a16_exact_known_answer(cuda_device, rng):
    """Small integers and power-of-two scales: every intermediate is exact, so the
    fp16 result must equal the exact value bit for bit."""
    M, N, K = 96, 384, 256
    A = rng.integers(-3, 4, (M, K)).astype(np.float16)
    q = rng.integers(-4, 5, (N, K)).astype(np.int8)
    q[0, :] = 127
    q[1, :] = -127
    s = (2.0 ** rng.integers(-10, -4, N)).astype(np.float16)
    C = nb.matmul(to_dev(A, cuda_device), to_dev(q, cuda_device), to_dev(s, cuda_device)).cpu().numpy()
    exact = ref.w8a16_ref(A, q, s)
    assert np.array_equal(C, exact.astype(np.float16))


@pytest.mark.parametrize("M,N,K", [(500, 600, 384), (1000, 256, 4096), (384, 1000, 1376)])
def test_w8a16_prefill_exact_known_answer(cuda_device, rng, M, N, K):
    """Prefill shapes (M >= 384) run the tensor-memory pair kernel: 256 x 192
    tiles, ragged in every dimension here.  Small integers keep every sum exact."""
    A = rng.integers(-3, 4, (M, K)).astype(np.float16)
    q = rng.integers(-4, 5, (N, K)).astype(np.int8)
    s = (2.0 ** rng.integers(-12, -6, N)).astype(np.float16)
    R = rng.integers(-8, 9, (M, N)).astype(np.float16)
    out = torch.zeros((M, N + 16), dtype=torch.float16, device=cuda_device)[:, 8:8 + N]
    nb.matmul(to_dev(A, cuda_device), to_dev(q, cuda_device), to_dev(s, cuda_device), out=out,
              residual=to_dev(R, cuda_device))
    exact = ref.w8a16_ref(A, q, s, residual=R)
    assert np.array_equal(out.cpu().numpy(), exact.astype(np.float16))


@pytest.mark.parametrize("M,N,K", [(40, 1000, 4096), (64, 384, 11008), (7, 4096, 128)])
def test_w8a16_decode_exact_known_answer(cuda_device, rng, M, N, K):
    """Decode shapes (M <= 64) run the stream-K kernel, whose tiles are cut
    between CTAs and summed from fp32 partials.  With small integers every
    partial sum is an exact fp32 integer, so any cut must give the exact value."""
    A = rng.integers(-3, 4, (M, K)).astype(np.float16)
    q = rng.integers(-4, 5, (N, K)).astype(np.int8)
    s = (2.0 ** rng.integers(-12, -6, N)).astype(np.float16)
    R = rng.integers(-8, 9, (M, N)).astype(np.float16)
    C = nb.matmul(to_dev(A, cuda_device), to_dev(q, cuda_device), to_dev(s, cuda_device),
                  residual=to_dev(R, cuda_device)).cpu().numpy()
    exact = ref.w8a16_ref(A, q, s, residual=R)
    assert np.array_equal(C, exact.astype(np.float16))


@pytest.mark.parametrize("M,N,K", [(64, 12288, 4096), (32, 22016, 4096), (64, 4096, 11008)])
def test_w8a16_decode_repeatable(cuda_device, M, N, K):
    """Tiles cut between CTAs are summed by whichever piece arrives last; the
    sum must not depend on which one that was, nor race with the pieces'
    stores: eight back-to-back calls give the same bits, within tolerance."""
    g = torch.Generator(device=cuda_device).manual_seed(M + N)
    q = torch.randint(-127, 128, (N, K), generator=g, device=cuda_device, dtype=torch.int8)
    s = (torch.rand(N, generator=g, device=cuda_device) * 1e-3 + 1e-3).half()
    A = torch.randn((M, K), generator=g, device=cuda_device).half()
    ref = (A.float() @ q.float().t()) * s.float()[None, :]
    first = nb.matmul(A, q, s)
    assert ((first.float() - ref).abs().max() / ref.abs().max()).item() <= TOL
    for _ in range(7):
        assert torch.equal(nb.matmul(A, q, s), first)


def test_w8a16_decode_shapes_share_one_workspace(cuda_device):
    """A decode layer's GEMMs (different N and K) run back to back on one
    workspace: the tile counters of one shape must not be disturbed by another
    shape's partial sums.  Run the sequence twice."""
    g = torch.Generator(device=cuda_device).manual_seed(9)
    shapes = [(2, 1024, 512), (2, 512, 512), (2, 2752, 512), (2, 512, 1376), (5, 300, 4096), (64, 130, 256)]
    mats = []
    for M, N, K in shapes:
        q = torch.randint(-127, 128, (N, K), generator=g, device=cuda_device, dtype=torch.int8)
        s = (torch.rand(N, generator=g, device=cuda_device) * 1e-3 + 1e-3).half()
        A = torch.randn((M, K), generator=g, device=cuda_device).half()
        mats.append((A, q, s, (A.float() @ q.float().t()) * s.float()[None, :]))
    for _ in range(2):
        for A, q, s, ref in mats:
            C = nb.matmul(A, q, s).float()
            assert ((C - ref).abs().max() / ref.abs().max()).item() <= TOL


def test_w8a16_decode_strided_alpha(cuda_device, rng):
    M, N, K = 20, 700, 1024
    A = rng.standard_normal((M, K)).astype(np.float16)
    q = rng.integers(-127, 128, (N, K)).astype(np.int8)
    s = (rng.uniform(0.5, 2, N) * 1e-3).astype(np.float16)
    R = rng.standard_normal((M, N)).astype(np.float16)
    out = torch.zeros((M, N + 40), dtype=torch.float16, device=cuda_device)[:, 16:16 + N]
    nb.matmul(to_dev(A, cuda_device), to_dev(q, cuda_device), to_dev(s, cuda_device), out=out,
              residual=to_dev(R, cuda_device), alpha=0.25)
    got = out.float().cpu().numpy()
    assert ref.rel_err(got, ref.w8a16_ref(A, q, s, residual=R, alpha=0.25)) <= TOL
    full = torch.zeros((M, N + 40), dtype=torch.float16, device=cuda_device)
    full[:, 16:16 + N] = out
    assert not full[:, :16].any() and not full[:, 16 + N:].any()  # nothing written outside the view


def test_w8a16_split_k_deterministic(cuda_device, rng):
    M, N, K = 64, 4096, 4096  # decode shape: split-K partials + reduction
    A = to_dev(rng.standard_normal((M, K)).astype(np.float16), cuda_device)
    q = to_dev(rng.integers(-127, 128, (N, K)).astype(np.int8), cuda_device)
    s = to_dev((np.ones(N) * 1e-3).astype(np.float16), cuda_device)
    c1 = nb.matmul(A, q, s)
    c2 = nb.matmul(A, q, s)
    assert torch.equal(c1, c2)


def test_w8a16_full_size_against_torch_fp32(cuda_device):
    """Gate|up projection of the Llama-7B layer at prefill size vs a torch fp32
    reference of the same op on the dequantised weights."""
    g = torch.Generator(device=cuda_device).manual_seed(7)
    M, N, K = 2048, 22016, 4096
    W = torch.randn((K, N), generator=g, device=cuda_device) * 0.02
    q, s = nb.quantize_w8(W)
    del W
    A = torch.randn((M, K), generator=g, device=cuda_device).half()
    C = nb.matmul(A, q, s).float()
    ref32 = (A.float() @ q.float().t()) * s.float()[None, :]
    e = ((C - ref32).abs().max() / ref32.abs().max()).item()
    assert e <= TOL
    assert torch.isfinite(C).all()


def test_f16_matmul_against_npu_matmul(cuda_device, examples):
    """fp16 weights: the reference's own matmul example (test_matmul.py, 8x64 @ 64x64)."""
    A, B = examples["matmul_A"], examples["matmul_B"]
    C = nb.matmul(to_dev(A.astype(np.float16), cuda_device), to_dev(B.T.astype(np.float16), cuda_device))
    got = C.float().cpu().numpy()
    assert ref.rel_err(got, examples["matmul_npu"]) <= TOL
    # fp16 store of an fp32 accumulation: nearly every element is byte-identical
    assert np.mean(got == examples["matmul_npu"]) > 0.95


def test_invalid_shapes_raise(cuda_device):
    A = torch.zeros((4, 24), dtype=torch.float16, device=cuda_device)
    q = torch.zeros((8, 24), dtype=torch.int8, device=cuda_device)
    with pytest.raises(ValueError):
        nb.matmul(A, q)  # K = 24 is not a multiple of 16
    with pytest.raises(ValueError):
        nb.matmul(A, torch.zeros((8, 16), dtype=torch.int8, device=cuda_device))  # K mismatch


@pytest.mark.parametrize("M,F,K", [(32, 11008, 4096), (64, 2752, 4096), (32, 1376, 4096), (2048, 1376, 4096),
                                   (300, 500, 272), (5, 64, 64), (17, 4100, 1024)])
def test_matmul_swiglu_equals_matmul_then_swiglu(cuda_device, M, F, K):
    """The fused gate|up + SwiGLU gives the bits of the two separate ops on the
    same interleaved weights (matmul, then swiglu on its even / odd columns):
    stream-K (M <= 64, 2F >= 8192), the pair kernel with and without split-K,
    ragged shapes.  (Against the [gate | up] layout the stream-K kernel cuts a
    row's K range at other places, so only the pair kernel matches bit for bit
    there; the oracle test below bounds both.)"""
    g = torch.Generator(device=cuda_device).manual_seed(M + F + K)
    W = torch.randn((K, 2 * F), generator=g, device=cuda_device) * 0.02
    q, s = nb.quantize_w8(W)
    del W
    A = torch.randn((M, K), generator=g, device=cuda_device).half()
    qi, si = nb.interleave_gate_up(q, s)
    gu = nb.matmul(A, qi, si)
    ref_out = nb.swiglu(gu[:, 0::2].contiguous(), gu[:, 1::2].contiguous())
    if M > 64:  # pair kernel: per-row sums independent of the row order
        assert torch.equal(ref_out, nb.swiglu(nb.matmul(A, q, s)))
    out = torch.full((M, F + 8), 7.0, dtype=torch.float16, device=cuda_device)
    nb.matmul_swiglu(A, qi, si, out=out[:, :F])
    assert torch.equal(out[:, :F], ref_out)
    assert bool((out[:, F:] == 7.0).all())  # nothing written past the F columns


def test_matmul_swiglu_against_oracle(cuda_device, rng):
    """Against the float64 oracle of the FFN's first half (llama_layer.py:143-150)."""
    M, F, K = 40, 300, 512
    A = rng.standard_normal((M, K)).astype(np.float16)
    W = (rng.standard_normal((K, 2 * F)) * 0.05).astype(np.float32)
    q, s = ref.quantize_w8(W)
    gu = ref.w8a16_ref(A, q, s).astype(np.float16).astype(np.float64)
    want = ref.silu_mul_ref(gu[:, :F], gu[:, F:])
    qi, si = nb.interleave_gate_up(to_dev(q, cuda_device), to_dev(s, cuda_device))
    got = nb.matmul_swiglu(to_dev(A, cuda_device), qi, si).float().cpu().numpy()
    assert ref.rel_err(got, want) <= TOL


# ------------------------------------------------ RMSNorm folded into the decode GEMMs

@pytest.mark.parametrize("M,N,K", [(32, 12288, 4096), (7, 1024, 512), (64, 4096, 4096), (1, 512, 1376)])
def test_matmul_rms_consumer_against_oracle(cuda_device, rng, M, N, K):
    """matmul_rms(rmsnorm_parts(h)) = RMSNorm(h) then the W8A16 projection
    (legalize.py:30-47 then npu.py:41-47), against the float64 oracle, and
    close to the unfused pair of launches."""
    h = (rng.standard_normal((M, K)) * 3).astype(np.float16)
    gam = (1 + 0.1 * rng.standard_normal(K)).astype(np.float16)
    W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    q, s = ref.quantize_w8(W)
    hd, gd, qd, sd = (to_dev(a, cuda_device) for a in (h, gam, q, s))
    g, ss = nb.rmsnorm_parts(hd, gd)
    got = nb.matmul_rms(g, qd, sd, rs=(ss, K), eps=1e-5).float().cpu().numpy()
    want = ref.w8a16_ref(ref.rmsnorm_ref(h, gam, 1e-5).astype(np.float16), q, s)
    assert ref.rel_err(got, want) <= TOL
    unfused = nb.matmul(nb.rmsnorm(hd, gd, 1e-5), qd, sd).float().cpu().numpy()
    assert ref.rel_err(got, unfused) <= 2e-3


def test_rmsnorm_parts_exact(cuda_device, rng):
    """g = fp16(x * gamma) bit for bit; ss = the sums of x^2 over every 32 columns."""
    x = (rng.standard_normal((5, 4096)) * 2).astype(np.float16)
    gam = rng.standard_normal(4096).astype(np.float16)
    g, ss = nb.rmsnorm_parts(to_dev(x, cuda_device), to_dev(gam, cuda_device))
    assert np.array_equal(g.cpu().numpy(), (x.astype(np.float32) * gam.astype(np.float32)).astype(np.float16))
    want = (x.astype(np.float64) ** 2).reshape(5, 128, 32).sum(-1).T
    assert np.allclose(ss.cpu().numpy(), want, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("M,N,K", [(32, 4096, 4096), (32, 4096, 11008), (13, 512, 512), (64, 1024, 1376)])
def test_matmul_rms_producer_outputs(cuda_device, rng, M, N, K):
    """The producer form: C = fp16(A Wq^T s + R) as matmul(residual=R) on the
    stream-K kernel, G = fp16(C * gamma) bit for bit from C, and the column
    sums of C^2 -- which a consumer call turns into the RMSNorm of C."""
    A = rng.standard_normal((M, K)).astype(np.float16)
    R = rng.standard_normal((M, N)).astype(np.float16)
    gam = (1 + 0.1 * rng.standard_normal(N)).astype(np.float16)
    W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    q, s = ref.quantize_w8(W)
    Ad, Rd, gd, qd, sd = (to_dev(a, cuda_device) for a in (A, R, gam, q, s))
    C, G, ss = nb.matmul_rms(Ad, qd, sd, residual=Rd, gamma=gd)
    Cn = C.float().cpu().numpy()
    assert ref.rel_err(Cn, ref.w8a16_ref(A, q, s, residual=R)) <= TOL
    assert torch.equal(G, (C.float() * gd.float()).half())
    want = (Cn.astype(np.float64) ** 2).reshape(M, N // 32, 32).sum(-1).T
    assert np.allclose(ss.cpu().numpy()[:, :M], want, rtol=1e-5, atol=1e-5)
    # the folded pair equals RMSNorm(C) then the next projection, within tolerance
    W2 = (rng.standard_normal((N, 256)) * 0.02).astype(np.float32)
    q2, s2 = ref.quantize_w8(W2)
    nxt = nb.matmul_rms(G, to_dev(q2, cuda_device), to_dev(s2, cuda_device), rs=(ss, N), eps=1e-6)
    want2 = ref.w8a16_ref(ref.rmsnorm_ref(Cn.astype(np.float16), gam, 1e-6).astype(np.float16), q2, s2)
    assert ref.rel_err(nxt.float().cpu().numpy(), want2) <= TOL


def test_matmul_rms_swiglu_against_oracle(cuda_device, rng):
    """Consumer form with SwiGLU: RMSNorm -> gate|up -> silu(g) * u (llama_layer.py:139-150)."""
    M, F, K = 32, 688, 512
    h = (rng.standard_normal((M, K)) * 2).astype(np.float16)
    gam = (1 + 0.1 * rng.standard_normal(K)).astype(np.float16)
    W = (rng.standard_normal((K, 2 * F)) * 0.05).astype(np.float32)
    q, s = ref.quantize_w8(W)
    hn = ref.rmsnorm_ref(h, gam, 1e-5).astype(np.float16)
    gu = ref.w8a16_ref(hn, q, s).astype(np.float16).astype(np.float64)
    want = ref.silu_mul_ref(gu[:, :F], gu[:, F:])
    qi, si = nb.interleave_gate_up(to_dev(q, cuda_device), to_dev(s, cuda_device))
    g, ss = nb.rmsnorm_parts(to_dev(h, cuda_device), to_dev(gam, cuda_device))
    got = nb.matmul_rms(g, qi, si, swiglu=True, rs=(ss, K), eps=1e-5).float().cpu().numpy()
    assert ref.rel_err(got, want) <= TOL


def test_matmul_rms_rejects_many_tokens(cuda_device):
    A = torch.zeros((65, 512), dtype=torch.float16, device=cuda_device)
    q = torch.zeros((512, 512), dtype=torch.int8, device=cuda_device)
    s = torch.ones(512, dtype=torch.float16, device=cuda_device)
    with pytest.raises(nb.NpubError):
        nb.matmul_rms(A, q, s)


@pytest.mark.parametrize("M,N,K", [(32, 4096, 4096), (17, 3072, 3072), (32, 2048, 4096), (5, 4096, 11008),
                                   (64, 4096, 4096)])
def test_stream_k_cluster_split_against_oracle(cuda_device, rng, M, N, K):
    """Matrices of few 128-row tiles run as one cluster per tile (2-8 CTAs
    splitting K, the pieces summed in the finisher's shared memory): against
    the oracle, with a residual, and bit-identical from call to call."""
    A = rng.standard_normal((M, K)).astype(np.float16)
    R = rng.standard_normal((M, N)).astype(np.float16)
    W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    q, s = ref.quantize_w8(W)
    Ad, Rd, qd, sd = (to_dev(a, cuda_device) for a in (A, R, q, s))
    got = nb.matmul_rms(Ad, qd, sd, residual=Rd)
    again = nb.matmul_rms(Ad, qd, sd, residual=Rd)
    assert torch.equal(got, again)
    assert ref.rel_err(got.float().cpu().numpy(), ref.w8a16_ref(A, q, s, residual=R)) <= TOL
    if M <= 32:
        plain = nb.matmul(Ad, qd, sd).float().cpu().numpy()
        assert ref.rel_err(plain, ref.w8a16_ref(A, q, s)) <= TOL

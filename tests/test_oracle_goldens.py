"""The oracle against the reference's golden vectors (CPU).

* 55 ISA example traces (_poc/goldens/*.txt, captured from the original cmodel
  binary): the C restatement must reproduce each trace byte for byte, the way
  the reference's _poc/verify_all.sh checks its simulator.
* The reference's example scripts (b_program_examples/test_*.py,
  llama_layer.py): the numpy restatements must reproduce the scripts' own
  python references, and the emitted programs run on the C restatement must
  reproduce the scripts' NPU outputs.
"""
import hashlib
import json
import os

import numpy as np
import pytest

from oracle import cmodel, emit, ref

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _isa():
    with open(os.path.join(GOLDEN, "isa_goldens.json")) as f:
        return json.load(f)


ISA = _isa()


def ramp():
    return np.arange(8192).astype(np.float16)


@pytest.mark.parametrize("prog", ISA["programs"], ids=[p["name"] for p in ISA["programs"]])
def test_isa_golden_trace(prog):
    words = np.zeros(prog["nwords"], dtype=np.uint32)
    words[: len(prog["words"])] = prog["words"]
    m = cmodel.Machine(ramp(), gcap=1 << 16)
    _, trace = m.execute(words, ISA["maxrun"], trace=True, gbytes=ISA["gbytes"], pbytes=ISA["pbytes"])
    assert len(trace.splitlines()) == prog["lines"]
    assert hashlib.sha256(trace.encode()).hexdigest() == prog["sha256"], prog["name"]


@pytest.mark.parametrize("prog", ISA["programs"][::11], ids=[p["name"] for p in ISA["programs"][::11]])
def test_isa_golden_trace_reference_simulator(prog):
    if not cmodel.have_mysim():
        pytest.skip("reference simulator not built here")
    words = np.zeros(prog["nwords"], dtype=np.uint32)
    words[: len(prog["words"])] = prog["words"]
    _, trace = cmodel.run_mysim(words, ramp(), 8192, maxrun=ISA["maxrun"], capture_trace=True)
    assert hashlib.sha256(trace.encode()).hexdigest() == prog["sha256"], prog["name"]


def test_ramp_fp16_store_rounding():
    # G[i] = fp16(i): integers above 2048 round to even multiples of 2, 4, ...
    g = cmodel.f32_to_f16_bits(np.arange(8192, dtype=np.float32)).view(np.float16)
    assert np.array_equal(g, ramp())


def test_example_matmul(examples):
    A, B = examples["matmul_A"], examples["matmul_B"]
    assert np.array_equal(ref.matmul_f16_pyref(A, B), examples["matmul_ref"])
    g = emit.GBuf()
    aA, aB, aC = g.alloc(A.size), g.alloc(B.size), g.alloc(A.shape[0] * B.shape[1])
    g.put(aA, A)
    g.put(aB, B)
    a = emit.Asm()
    emit.matmul(a, aA, aB, aC, A.shape[0], A.shape[1], B.shape[1])
    a.halt()
    out = cmodel.run_oracle(a.words, g.image(g.top), g.top)
    C = out[aC: aC + A.shape[0] * B.shape[1]].reshape(A.shape[0], B.shape[1]).astype(np.float32)
    assert np.array_equal(C, examples["matmul_npu"])


def test_example_rmsnorm(examples):
    X, W = examples["rmsnorm_X"], examples["rmsnorm_W"]
    assert np.array_equal(ref.rmsnorm_npu_ref(X, W), examples["rmsnorm_ref"])
    words, gimg, a_out, gn = emit.rmsnorm_program(X, W)
    out = cmodel.run_oracle(words, gimg, gn, maxrun=len(words) + 1)
    got = out[a_out: a_out + X.size].reshape(X.shape).astype(np.float32)
    assert np.array_equal(got, examples["rmsnorm_npu"])
    # the script's own tolerance (test_rmsnorm.py:57)
    assert np.abs(got - examples["rmsnorm_ref"]).max() < 1e-2


def test_example_swiglu(examples):
    X, Wg, Wu, Wd = (examples[f"swiglu_{k}"] for k in ("X", "Wg", "Wu", "Wd"))
    G = ref.matmul_f16_pyref(X, Wg)
    U = ref.matmul_f16_pyref(X, Wu)
    H = ref.swiglu_npu_ref(G, U)
    assert np.array_equal(ref.matmul_f16_pyref(H, Wd), examples["swiglu_ref"])
    # the NPU program: float32 matmuls (mysim) around the exp/add/div/mul recipe
    Gn, Un = ref.matmul_f16_ref(X, Wg), ref.matmul_f16_ref(X, Wu)
    words, gimg, a_h, gn = emit.swiglu_program(Gn, Un)
    out = cmodel.run_oracle(words, gimg, gn, maxrun=len(words) + 1)
    Hn = out[a_h: a_h + H.size].reshape(H.shape).astype(np.float32)
    got = ref.matmul_f16_ref(Hn, Wd)
    assert np.array_equal(got, examples["swiglu_npu"])
    assert np.abs(got - examples["swiglu_ref"]).max() < 3e-2  # test_swiglu.py:51


def test_example_attention(examples):
    X, Wq, Wk, Wv, Wo = (examples[f"attention_{k}"] for k in ("X", "Wq", "Wk", "Wv", "Wo"))
    S, D = X.shape
    HD = Wq.shape[1]
    Q = ref.matmul_f16_ref(X, Wq)
    Kt = ref.matmul_f16_ref(Wk.T, X.T)
    V = ref.matmul_f16_ref(X, Wv)
    Sc = ref.f16(ref.matmul_f16_ref(Q, Kt) / np.float32(np.sqrt(HD)))
    words, gimg, a_p, gn = emit.softmax_program(Sc, causal=True)
    out = cmodel.run_oracle(words, gimg, gn, maxrun=len(words) + 1)
    P = out[a_p: a_p + S * S].reshape(S, S).astype(np.float32)
    got = ref.matmul_f16_ref(ref.matmul_f16_ref(P, V), Wo)
    assert np.array_equal(got, examples["attention_npu"])
    # and the float64 stable-softmax reference agrees within the script's tolerance
    f = ref.attention_ref(X @ Wq, X @ Wk, X @ Wv, 1, 1, HD) @ Wo
    assert np.abs(f - examples["attention_ref"]).max() < 2e-2


def _layer_weights(ex):
    SEQ, D, H, KV, HD, F = (int(v) for v in ex["layer_dims"])
    W = {"Wn1": ex["layer_Wn1"], "Wn2": ex["layer_Wn2"], "Wg": ex["layer_Wg"], "Wu": ex["layer_Wu"],
         "Wd": ex["layer_Wd"]}
    for h in range(H):
        W[f"Wq{h}"] = ex["layer_Wq"][h]
        W[f"Wo{h}"] = ex["layer_Wo"][h]
    for k in range(KV):
        W[f"Wk{k}"] = ex["layer_Wk"][k]
        W[f"Wv{k}"] = ex["layer_Wv"][k]
    return W, (SEQ, D, H, KV, HD, F)


def test_example_layer_float_reference(examples):
    W, (SEQ, D, H, KV, HD, F) = _layer_weights(examples)
    cos, sin = ref.rope_tables(SEQ, HD)
    y = ref.ref_layer(W, examples["layer_X"], H, KV, HD, 0.0, cos, sin)
    # the script's float reference (llama_layer.py:157-195), pure-python doubles
    assert np.abs(y - examples["layer_ref"]).max() < 1e-5
    # the NPU output of the script (mysim) is within its own check (llama_layer.py:199-205)
    assert ref.rel_err(examples["layer_npu"], examples["layer_ref"]) < 0.01


def test_rope_program_matches_float_rope(rng):
    S, HD = 8, 16
    Q = ref.f16(rng.uniform(-1, 1, (S, HD)))
    cos, sin = ref.rope_tables(S, HD)
    words, gimg, a_o, gn = emit.rope_program(Q, ref.f16(cos), ref.f16(sin))
    out = cmodel.run_oracle(words, gimg, gn, maxrun=len(words) + 1)
    got = out[a_o: a_o + Q.size].reshape(S, HD).astype(np.float32)
    exp = ref.rope_ref(Q, 1, HD, np.arange(S))
    assert np.abs(got - exp).max() < 1e-2

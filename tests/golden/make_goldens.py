"""Regenerate the golden fixtures of tests/golden/ from the reference tree.

Run where a checkout of the reference (KwanyoungCho/NPU_COMP) is available:

    python tests/golden/make_goldens.py --ref <reference root>

(or with NPU_COMP_REF=<reference root> in the environment).

It never copies reference sources into this repository.  It compiles and runs
the reference's own generators and simulator (outputs under oracle/_ref/ and a
temporary directory) and records only their outputs:

  isa_goldens.json   for each of the 55 ISA example programs under
                     b_program/inst_*/: the program words produced by its
                     w_support_program_mem_gen.cpp, the line count and sha256
                     of the golden trace _poc/goldens/<name>.txt (captured from
                     the original cmodel binary on the ramp G-buffer made by
                     c_hex_data/w_support_binary_data_gen.cpp).  The script
                     also asserts that our C restatement (oracle/isa_oracle.c)
                     and the reference simulator reproduce every trace.
  examples.npz       inputs and outputs of the reference's example scripts
                     b_program_examples/test_{matmul,rmsnorm,swiglu,attention}.py
                     and llama_layer.py, run as-is (on a copy, with mysim
                     built from _poc/mysim.cpp): the G-buffer results of the
                     NPU programs and the scripts' own python references.
  programs.npz       every program the example scripts hand to run(): the
                     program words and the initial G-buffer exactly as run()
                     wrote them, its gn / maxrun, and the simulator's
                     write-back (gout.bin) -- for the GPU program executor.
  w8a16_config1.npz  the single W8A16 matmul configuration (A [64,512] ~N(0,1),
                     W [512,512] ~N(0,0.02), numpy default_rng(0)) run through
                     the compiler-style 64-tiled program on the reference
                     simulator: C as fp16, with sha256 of the inputs.
  rope_tables.npz    the compiler's host RoPE tables (cos, sin, rotate_half
                     matrix) from d_compiler/npu_compiler/legalize.py's own
                     rope_tables(), for the Llama 3.2 3B layer (base 500000,
                     Llama-3 frequency scaling) and the reduced layer (base
                     10000); rows sampled over positions 0..4199.  legalize.py imports TVM's relax module at the top
                     but these functions only use numpy, so it is loaded with a
                     placeholder `tvm` module.
  --only rope        regenerates that file alone.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import runpy
import shutil
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import cmodel, emit, ref  # noqa: E402


def _gxx(src, out):
    os.makedirs(os.path.dirname(out), exist_ok=True)
    if not os.path.exists(out) or os.path.getmtime(src) > os.path.getmtime(out):
        subprocess.run(["g++", "-O2", "-std=c++17", src, "-o", out], check=True)
    return out


def ramp_gbuffer(refdir):
    exe = _gxx(os.path.join(refdir, "c_hex_data", "w_support_binary_data_gen.cpp"),
               os.path.join(ROOT, "oracle", "_ref", "gen", "gbuf_ramp"))
    with tempfile.TemporaryDirectory() as d:
        subprocess.run([exe], cwd=d, check=True, stdout=subprocess.DEVNULL)
        raw = open(os.path.join(d, "G_buffer_data.bin"), "rb").read()
    return raw


def isa_goldens(refdir):
    gbuf_raw = ramp_gbuffer(refdir)
    gbuf = np.frombuffer(gbuf_raw[: (len(gbuf_raw) // 2) * 2], dtype="<f2")
    assert len(gbuf_raw) == 16385 and np.array_equal(gbuf.astype(np.float32), np.arange(8192, dtype=np.float16)
                                                     .astype(np.float32)), "ramp G-buffer mismatch"
    out = []
    gold_dir = os.path.join(refdir, "_poc", "goldens")
    for fn in sorted(os.listdir(gold_dir)):
        name = fn[:-4]
        src = os.path.join(refdir, "b_program", name, "w_support_program_mem_gen.cpp")
        exe = _gxx(src, os.path.join(ROOT, "oracle", "_ref", "gen", name))
        with tempfile.TemporaryDirectory() as d:
            subprocess.run([exe], cwd=d, check=True, stdout=subprocess.DEVNULL)
            praw = open(os.path.join(d, "program_memory.bin"), "rb").read()
        assert len(praw) == 1025, (name, len(praw))
        words = np.frombuffer(praw[:1024], dtype="<u4")
        text = open(os.path.join(gold_dir, fn)).read()
        # our restatement; like _poc/verify_all.sh, the trace of the default
        # 30-instruction run is compared with the same number of golden lines
        m = cmodel.Machine(gbuf.astype(np.float16), gcap=1 << 16)
        _, trace = m.execute(words, 30, trace=True, gbytes=16385, pbytes=1025)
        mine = trace
        lines = text.splitlines(keepends=True)[: len(trace.splitlines())]
        golden = "".join(lines)
        assert mine == golden, f"C restatement differs from golden {name}"
        # the reference simulator rebuilt from source
        if cmodel.have_mysim():
            with tempfile.TemporaryDirectory() as d:
                open(os.path.join(d, "program_memory.bin"), "wb").write(praw)
                open(os.path.join(d, "G_buffer_data.bin"), "wb").write(gbuf_raw)
                r = subprocess.run([cmodel.MYSIM], cwd=d, capture_output=True, text=True, check=True)
            sim = r.stdout
            assert sim == golden, f"mysim differs from golden {name}"
        nz = int(np.max(np.nonzero(words)[0])) + 1 if words.any() else 0
        out.append({"name": name, "words": [int(w) for w in words[:nz]], "nwords": int(words.size),
                    "lines": len(lines), "sha256": hashlib.sha256(golden.encode()).hexdigest()})
    return out


_CAPTURE = """#!{python}
# Runs the reference simulator with the arguments run() gave, then keeps the
# program, the input G-buffer, the write-back and the arguments of the call.
import json, os, shutil, subprocess, sys
r = subprocess.run([{mysim!r}] + sys.argv[1:], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
d = os.path.join({cap!r}, "%03d" % len(os.listdir({cap!r})))
os.makedirs(d)
for f in ("program_memory.bin", "G_buffer_data.bin"):
    shutil.copy(f, d)
a = sys.argv[1:]
gout = a[a.index("--gout") + 1]
shutil.copy(gout, os.path.join(d, "gout.bin"))
json.dump(a, open(os.path.join(d, "args.json"), "w"))
sys.exit(r.returncode)
"""


def run_script(refdir, script, workdir, capture=None):
    """Run a reference example script as-is in a copy of its directory; return its
    globals.  With `capture` (a directory), every run() of the script leaves its
    program_memory.bin, G_buffer_data.bin, gout.bin and arguments there."""
    sdir = os.path.join(refdir, "b_program_examples")
    for f in ("npu.py", script):
        shutil.copy(os.path.join(sdir, f), workdir)
    if capture is None:
        shutil.copy(cmodel.MYSIM, os.path.join(workdir, "mysim"))
    else:
        os.makedirs(capture, exist_ok=True)
        with open(os.path.join(workdir, "mysim"), "w") as f:
            f.write(_CAPTURE.format(python=sys.executable, mysim=os.path.abspath(cmodel.MYSIM), cap=capture))
        os.chmod(os.path.join(workdir, "mysim"), 0o755)
    cwd = os.getcwd()
    sys.path.insert(0, workdir)
    try:
        os.chdir(workdir)
        for mod in ("npu",):
            sys.modules.pop(mod, None)
        import io
        import contextlib
        buf = io.StringIO()
        with contextlib.redirect_stdout(buf):
            g = runpy.run_path(os.path.join(workdir, script), run_name="__main__")
        g["__stdout__"] = buf.getvalue()
        return g
    finally:
        os.chdir(cwd)
        sys.path.remove(workdir)


def examples(refdir):
    res = {}
    with tempfile.TemporaryDirectory() as d:
        g = run_script(refdir, "test_matmul.py", d)
        res["matmul_A"] = np.array(g["A"], np.float32)
        res["matmul_B"] = np.array(g["B"], np.float32)
        res["matmul_npu"] = np.array(g["got"], np.float32).reshape(g["M"], g["N"])
        res["matmul_ref"] = np.array(g["exp"], np.float32).reshape(g["M"], g["N"])
    with tempfile.TemporaryDirectory() as d:
        g = run_script(refdir, "test_rmsnorm.py", d)
        res["rmsnorm_X"] = np.array(g["X"], np.float32)
        res["rmsnorm_W"] = np.array(g["W"], np.float32)
        res["rmsnorm_npu"] = np.array(g["got"], np.float32)
        res["rmsnorm_ref"] = np.array(g["exp"], np.float32)
    with tempfile.TemporaryDirectory() as d:
        g = run_script(refdir, "test_swiglu.py", d)
        for k in ("X", "Wg", "Wu", "Wd"):
            res[f"swiglu_{k}"] = np.array(g[k], np.float32)
        res["swiglu_npu"] = np.array(g["got"], np.float32).reshape(g["SEQ"], g["D"])
        res["swiglu_ref"] = np.array(g["Outr"], np.float32).reshape(g["SEQ"], g["D"])
    with tempfile.TemporaryDirectory() as d:
        g = run_script(refdir, "test_attention.py", d)
        for k in ("X", "Wq", "Wk", "Wv", "Wo"):
            res[f"attention_{k}"] = np.array(g[k], np.float32)
        res["attention_npu"] = np.array(g["got"], np.float32).reshape(g["SEQ"], g["D"])
        res["attention_ref"] = np.array(g["Outr"], np.float32).reshape(g["SEQ"], g["D"])
    with tempfile.TemporaryDirectory() as d:
        g = run_script(refdir, "llama_layer.py", d)
        H, KV = g["H"], g["KV"]
        res["layer_X"] = np.array(g["X"], np.float32)
        res["layer_Wn1"] = np.array(g["Wn1"], np.float32)
        res["layer_Wn2"] = np.array(g["Wn2"], np.float32)
        res["layer_Wq"] = np.array(g["Wq"], np.float32)      # [H, D, HD]
        res["layer_Wk"] = np.array(g["Wk"], np.float32)      # [KV, D, HD]
        res["layer_Wv"] = np.array(g["Wv"], np.float32)
        res["layer_Wo"] = np.array(g["Wo"], np.float32)      # [H, HD, D]
        res["layer_Wg"] = np.array(g["Wg"], np.float32)
        res["layer_Wu"] = np.array(g["Wu"], np.float32)
        res["layer_Wd"] = np.array(g["Wd"], np.float32)
        res["layer_cos"] = np.array(g["COS"], np.float32)
        res["layer_sin"] = np.array(g["SIN"], np.float32)
        res["layer_npu"] = np.array(g["got"], np.float32).reshape(g["SEQ"], g["D"])
        res["layer_ref"] = np.array(g["exp"], np.float32).reshape(g["SEQ"], g["D"])
        res["layer_dims"] = np.array([g["SEQ"], g["D"], H, KV, g["HD"], g["F"]], np.int64)
    return res


EXAMPLE_SCRIPTS = ("test_matmul.py", "test_rmsnorm.py", "test_swiglu.py", "test_attention.py", "llama_layer.py")


def programs(refdir):
    """The programs the reference's example scripts build and hand to run(),
    as run() wrote them (program words, initial G-buffer), with the arguments
    and the simulator's write-back: arrays <script>_<i>_{words,gin,gout,gn,maxrun}."""
    res = {}
    for script in EXAMPLE_SCRIPTS:
        name = script[:-3]
        with tempfile.TemporaryDirectory() as d, tempfile.TemporaryDirectory() as cap:
            run_script(refdir, script, d, capture=cap)
            for i, sub in enumerate(sorted(os.listdir(cap))):
                c = os.path.join(cap, sub)
                args = json.load(open(os.path.join(c, "args.json")))
                praw = open(os.path.join(c, "program_memory.bin"), "rb").read()
                graw = open(os.path.join(c, "G_buffer_data.bin"), "rb").read()
                oraw = open(os.path.join(c, "gout.bin"), "rb").read()
                k = f"{name}_{i}"
                res[k + "_words"] = np.frombuffer(praw[: len(praw) // 4 * 4], dtype="<u4").astype(np.uint32)
                res[k + "_gin"] = np.frombuffer(graw[: len(graw) // 2 * 2], dtype="<f2").astype(np.float16)
                res[k + "_gout"] = np.frombuffer(oraw[: len(oraw) // 2 * 2], dtype="<f2").astype(np.float16)
                res[k + "_gn"] = np.int64(args[args.index("--gn") + 1])
                res[k + "_maxrun"] = np.int64(args[args.index("--run") + 1])
    return res


def config1():
    rng = np.random.default_rng(0)
    A = rng.standard_normal((64, 512)).astype(np.float16)
    W = (rng.standard_normal((512, 512)) * 0.02).astype(np.float32)
    q, s = ref.quantize_w8(W)
    words, gimg, ca, gn = emit.w8a16_program(A, ref.dequant_f16(q, s))
    C = cmodel.run_mysim(words, gimg, gn, maxrun=len(words) + 1)[ca: ca + 64 * 512].reshape(64, 512)
    return {"C_mysim": C.astype(np.float16), "instructions": np.int64(len(words)),
            "sha_A": hashlib.sha256(A.tobytes()).hexdigest(), "sha_W": hashlib.sha256(W.tobytes()).hexdigest()}


def rope_tables(refdir):
    """cos/sin/rot from the reference compiler's rope_tables (legalize.py:67-85)."""
    import importlib.util
    import types
    tvm = types.ModuleType("tvm")
    tvm.relax = types.ModuleType("tvm.relax")
    saved = {k: sys.modules.get(k) for k in ("tvm", "tvm.relax")}
    sys.modules["tvm"], sys.modules["tvm.relax"] = tvm, tvm.relax
    try:
        spec = importlib.util.spec_from_file_location(
            "ref_legalize", os.path.join(refdir, "d_compiler", "npu_compiler", "legalize.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v
    out = {}
    for name, seq, hd, base, scaled in (("llama3", 4200, 128, 500000.0, True), ("reduced", 8, 16, 10000.0, False),
                                        ("hd128", 4200, 128, 10000.0, False)):
        cos, sin, rot = mod.rope_tables(seq, hd, base=base, llama3_scaling=scaled)
        rows = np.unique(np.concatenate([np.arange(min(seq, 16)), np.arange(0, seq, 131), np.arange(seq - 8, seq)]))
        out[f"{name}_rows"] = rows
        out[f"{name}_cos"], out[f"{name}_sin"], out[f"{name}_rot"] = cos[rows], sin[rows], rot
        out[f"{name}_args"] = np.array([seq, hd, base, float(scaled)])
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("NPU_COMP_REF"),
                    help="root of the reference checkout (default: $NPU_COMP_REF)")
    ap.add_argument("--only", choices=["programs", "rope"], default=None, help="regenerate one fixture file only")
    a = ap.parse_args()
    if not a.ref:
        ap.error("the reference root is required: --ref <dir> or NPU_COMP_REF=<dir>")
    if a.only == "rope":
        np.savez_compressed(os.path.join(HERE, "rope_tables.npz"), **rope_tables(a.ref))
        print("wrote rope_tables.npz")
        return
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), f"REF={a.ref}"], check=True)
    progs = programs(a.ref)
    np.savez_compressed(os.path.join(HERE, "programs.npz"), **progs)
    if a.only == "programs":
        print(f"wrote programs.npz ({len(progs) // 5} program runs)")
        return
    gold = isa_goldens(a.ref)
    with open(os.path.join(HERE, "isa_goldens.json"), "w") as f:
        json.dump({"gbuf": "ramp G[i] = fp16(i), i < 8192 (c_hex_data/w_support_binary_data_gen.cpp)",
                   "maxrun": 30, "gbytes": 16385, "pbytes": 1025, "programs": gold}, f, indent=0)
    np.savez_compressed(os.path.join(HERE, "examples.npz"), **examples(a.ref))
    np.savez_compressed(os.path.join(HERE, "rope_tables.npz"), **rope_tables(a.ref))
    c1 = config1()
    np.savez_compressed(os.path.join(HERE, "w8a16_config1.npz"), C_mysim=c1["C_mysim"],
                        instructions=c1["instructions"], sha_A=np.array(c1["sha_A"]), sha_W=np.array(c1["sha_W"]))
    print(f"wrote {len(gold)} ISA goldens, examples.npz, w8a16_config1.npz")


if __name__ == "__main__":
    main()

"""Oracle for the W8A16 / Llama-layer hot path -- TEST INFRASTRUCTURE ONLY.

This package is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
it; ``npu_comp_b200`` never does, and its CUDA path fails loudly instead of
falling back here.

Contents
--------
``isa_oracle.c`` / ``cmodel.py``
    C restatement of the reference cmodel ``_poc/mysim.cpp`` (fp16 rounding,
    float32 compute, the instruction loop and its stdout trace), plus a runner
    for the reference binary itself, built from ``_poc/mysim.cpp`` into
    ``oracle/_ref/mysim`` by ``oracle/Makefile``.
``emit.py``
    numpy-only instruction emitter and the program builders the reference
    compiler would produce (tiled matmul ``d_compiler/npu_compiler/codegen.py:59-108``,
    chunked elementwise ``codegen.py:160-177``, legalize recipes
    ``d_compiler/npu_compiler/legalize.py:20-149``, layer graph
    ``d_compiler/npu_compiler/model.py:64-112``).
``ref.py``
    numpy restatements of the reference's python goldens (per-save fp16
    rounding references in ``b_program_examples/test_*.py``,
    ``tiled_fp16_ref`` of ``d_compiler/tests/test_tiling.py:37-47``, float64
    ``ref_layer`` of ``d_compiler/npu_compiler/model.py:115-157``) and of the
    W8A16 quantisation, which the reference does not have (parity of that part
    is unpinned by any reference test).

Pinning: the C restatement reproduces all 55 golden traces byte for byte and
agrees with the reference binary on every program the tests run; the numpy
references reproduce the reference scripts' outputs recorded under
``tests/golden/`` by ``tests/golden/make_goldens.py``.
"""

"""TEST INFRASTRUCTURE ONLY -- the CPU oracle of the b200 non-GEMM op path.

Nothing in the product imports this package.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may use it,
and only as the checker (or the timed CPU baseline), never as the thing that
is measured on the GPU or shipped.

Contents
--------
``ops``        numpy restatement of every op on the path, in two flavours:
               ``golden`` (fp64 math, one final rounding: the "fp32-accumulated
               result" the bf16/f16 tolerances are stated against) and
               ``chain`` (fp32 math rounded after every step exactly where the
               reference's op-by-op chain on the flagos device rounds).
``hf_chain``   the reference's own CPU path: the HuggingFace formulas
               (transformers 5.5.0, models/qwen3/modeling_qwen3.py) over torch
               2.11 CPU aten ops.  Used to generate the golden fixtures under
               tests/golden/ and as the timed CPU baseline.
``oracle.c``   plain-C restatement of the exact integer / index reductions
               (int32 -> int64 sums, first-index argmax over bf16 bits),
               built to ``oracle/_build/liboracle.so`` by ``oracle/Makefile``.
``native``     ctypes loader for liboracle.so.

Pinning: ``ops`` is checked against the fixtures in tests/golden/, which
``tests/golden/make_golden.py`` produced by running the reference's own
formulas (``hf_chain``) on torch CPU with seeded inputs.
"""

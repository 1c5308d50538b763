"""TEST INFRASTRUCTURE ONLY: the CPU oracle of the decision hot path.

A CPU restatement of the reference's algorithm (firelex/jeff, runtime/python/src/jeff_runtime/engine/ and the
transformers Qwen3.5 model it runs), used as the checker of the CUDA path. Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg (and its `--impl reference` arm) may import it. The product (package jeff_b200) never
imports, calls or links anything here, and has no CPU fallback.

- int4_ref: numpy restatement of the int4 kernel layout, pack/unpack and dequantisation (bit-exact integer work).
- model_ref: torch-CPU restatement of every kernel of the pass and of the whole batched forward, with the fast path's
  bfloat16 rounding points (or none, `exact=True`, to compare with the reference's float32 standard path).

Pinning: tests/golden/ holds vectors produced by running the reference's own code on a machine with a checkout of
the reference (tests/golden/make_golden.py, pointed at it by $JEFF_REFERENCE): its int4 packer/dequantiser, its PrefixShapes layout, the
transformers torch_chunk_gated_delta_rule (the standard path's scan) and the transformers Qwen3.5 text model forward
on seeded synthetic weights. tests/test_oracle_golden.py checks this oracle against them."""

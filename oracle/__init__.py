"""CPU oracle of the SheetSage2-Refined decode step — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, what the reference computes on the decode
hot path: the batched greedy step of ``sheetsage2_refined/engine.py:294-357``
(the post-LN decoder of ``decoder.py:58-151`` fed one token per slot), the
token grammar of ``grammar.py:114-197`` and the slot life cycle of
``engine.py:176-262``.  It exists to check the CUDA engine, nothing else:

* only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU
  baseline and its ``--impl reference`` arm) may import it;
* the product package ``sheetsage2_refined_b200`` never imports it and has no
  CPU fallback.

Two numerics modes are restated:

* ``"fp32"`` — the reference's CPU path (engine.py:69-70: float32 weights,
  no autocast).  Pinned against golden vectors produced by running the
  reference itself (``tests/golden/make_golden.py``).
* ``"bf16"`` — the reference's CUDA path (engine.py:12-15,118-123,297-315):
  Linear inputs, weights and outputs rounded to bfloat16 with float32
  accumulation, K/V cached in bfloat16, attention scores rounded to bfloat16
  before the 1/8 scale, softmax in float32 then rounded to bfloat16, residual
  sums and LayerNorm in float32, GELU on bfloat16, logits rounded to bfloat16.
  Its rounding points are the ones the reference's bf16 autocast applies; it
  is checked against the fp32 mode within the logit tolerance and is the
  comparison target of the GPU tests.
"""

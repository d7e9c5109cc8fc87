"""CPU oracle for the silogic logic-gate-network hot path -- TEST INFRASTRUCTURE ONLY.

This package restates the reference algorithm on the CPU so that the CUDA path
in ``silogic_b200`` can be checked against it.  It is imported only by
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py``; the product never imports, links or calls it.

* :mod:`oracle.spec` -- turns a constructor call + ``state_dict`` into a plain
  per-layer description (wiring, truth tables, soft parameters), following the
  reference constructors ``silogic/models.py:23-104,153-293`` and
  ``silogic/layers.py:20-135,226-541``.
* :mod:`oracle.hard` -- numpy bit-packed evaluation (64 samples per uint64 word),
  restating ``silogic/bitpacking/ops.py``, ``convert.py`` and ``packed_layer.py``.
* :mod:`oracle.soft` -- fp32 torch restatement of the soft (relaxed) forward whose
  gradients come from torch autograd, restating ``silogic/nodes.py``,
  ``connectomes.py``, ``layers.py``, ``heads.py`` and ``encoders.py``.

Pinning: every function here is checked in ``tests/test_oracle.py`` against the
golden fixtures in ``tests/golden/`` that ``tests/golden/make_golden.py``
produced by running the reference itself (hard counts bit-exact, soft logits and
gradients to 1e-5).
"""

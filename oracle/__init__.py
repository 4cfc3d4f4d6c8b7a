"""CPU oracle for the B200 hot path -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.

This package restates, on the CPU, the algorithms of the reference (JESUSROYETH/rf-detr-jax)
for the three pieces of the training hot path:

* ``oracle.msda``    -- the multi-scale deformable-attention sampler, forward and backward
  (reference ``src/rfdetr_jax/models/ops.py:64-134,208-292``; gradient formulas
  ``src/rfdetr_jax/models/deform_pallas.py:56-120``).
* ``oracle.topk``    -- the two-stage query selection: class max, ``lax.top_k`` and
  ``select_rows`` (``src/rfdetr_jax/models/transformer.py:694-706``,
  ``src/rfdetr_jax/models/layers.py:225-244``).
* ``oracle.matcher`` -- the matching cost and the padded Hungarian solve
  (``src/rfdetr_jax/models/matcher.py:36-208``, ``src/rfdetr_jax/utilities/box_ops.py:27-75``).
* ``oracle/lsap.c``  -- a C restatement of SciPy's ``linear_sum_assignment`` (Crouse's shortest
  augmenting path), which the reference calls at ``matcher.py:173``.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference legs may
import anything from here, and only as the checker or the timed CPU baseline.  The product
(``rf-detr-jax_b200``) never imports, links or runs this package.

Pinning: the sampler restatement is checked against the reference's own known-answer tests
(``tests/test_ops.py:22-54``) and against ``torch.nn.functional.grid_sample`` -- the upstream
PyTorch op the reference's sampler reimplements (``ops.py:14-16``) -- forward and autograd
backward.  The LSAP restatement is checked bit-exactly against SciPy, which *is* the
reference's solver.  Top-k follows the documented ``jax.lax.top_k`` contract (descending, lower
index first on ties); JAX is not installed here, so that tie rule is pinned by the reference's
tests' semantics, not by running JAX.
"""

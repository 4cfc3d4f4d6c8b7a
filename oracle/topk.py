"""CPU oracle for the two-stage query selection -- TEST INFRASTRUCTURE.

Restates ``src/rfdetr_jax/models/transformer.py:694-706``:

* ``proposal_scores = logits.max(-1)`` (``:695``) -- a max over classes that propagates NaN;
* ``_, topk_indices = jax.lax.top_k(proposal_scores, topk)`` (``:696``) with
  ``topk = min(num_queries, positions)`` (``:694``);
* ``select_rows(values, topk_indices)`` (``src/rfdetr_jax/models/layers.py:225-244``).

``jax.lax.top_k`` returns the ``k`` largest entries in descending order; equal entries keep the
lower index first.  Ordering follows IEEE-754 totalOrder (``-NaN < -inf < ... < -0 < +0 < ...
< +inf < +NaN``), which is how XLA's TopK compares floats.  JAX is not installed here, so the
tie rule is restated from that contract rather than pinned by running JAX.
"""

from __future__ import annotations

import numpy as np


def total_order_key(scores: np.ndarray) -> np.ndarray:
    """Map float32 values to uint32 keys whose unsigned order is IEEE totalOrder."""
    bits = np.ascontiguousarray(scores, np.float32).view(np.uint32)
    negative = (bits >> 31).astype(bool)
    return np.where(negative, ~bits, bits | np.uint32(0x80000000)).astype(np.uint32)


def class_max(logits: np.ndarray) -> np.ndarray:
    """``logits.max(-1)`` (``transformer.py:695``), NaN-propagating."""
    return np.max(np.asarray(logits, np.float32), axis=-1)


def top_k(scores: np.ndarray, k: int):
    """``jax.lax.top_k(scores, k)``: descending values, lower index first on ties.

    Returns:
        ``(values float32 [..., k], indices int32 [..., k])``.
    """
    scores = np.asarray(scores, np.float32)
    if k < 0 or k > scores.shape[-1]:
        raise ValueError("k must be in [0, positions]")
    keys = total_order_key(scores).astype(np.int64)
    order = np.argsort(-keys, axis=-1, kind="stable")[..., :k]
    return np.take_along_axis(scores, order, axis=-1), order.astype(np.int32)


def select_rows(values: np.ndarray, indices: np.ndarray) -> np.ndarray:
    """``select_rows`` (``layers.py:225-244``): gather rows ``[..., N, C]`` at ``[..., K]``."""
    return np.take_along_axis(np.asarray(values), np.asarray(indices)[..., None].astype(np.int64), axis=-2)


def two_stage_select(logits: np.ndarray, num_queries: int):
    """Class max then top-k over proposals (``transformer.py:694-696``).

    Args:
        logits: ``[..., positions, classes]``.

    Returns:
        ``(scores [..., positions], topk_values [..., k], topk_indices int32 [..., k])``.
    """
    scores = class_max(logits)
    k = min(num_queries, scores.shape[-1])
    values, indices = top_k(scores, k)
    return scores, values, indices

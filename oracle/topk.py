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


def post_process(probabilities: np.ndarray, pred_boxes: np.ndarray, target_sizes: np.ndarray, num_classes: int,
                 num_select: int = 300):
    """The reference's ``post_process`` (``postprocess.py:37-51``) from already computed sigmoid
    probabilities ``[B, Q*C]``: top-k, query/label split, ``xyxy`` boxes (``box_ops.py:27-32``)
    scaled to ``(width, height)`` and clipped to the image."""
    batch = probabilities.shape[0]
    k = min(num_select, probabilities.shape[1])
    scores, indexes = top_k(probabilities, k)
    query_index = indexes // num_classes
    labels = (indexes % num_classes).astype(np.int32)
    b = np.asarray(pred_boxes, np.float32)
    cx, cy = b[..., 0], b[..., 1]
    w, h = np.clip(b[..., 2], 0.0, None), np.clip(b[..., 3], 0.0, None)
    xyxy = np.stack([cx - np.float32(0.5) * w, cy - np.float32(0.5) * h, cx + np.float32(0.5) * w,
                     cy + np.float32(0.5) * h], axis=-1).astype(np.float32)
    xyxy = np.take_along_axis(xyxy, query_index[..., None].astype(np.int64), axis=1)
    sizes = np.asarray(target_sizes)
    height, width = sizes[:, 0].astype(np.float32), sizes[:, 1].astype(np.float32)
    scale = np.stack([width, height, width, height], axis=1)[:, None, :]
    xyxy = np.clip(xyxy * scale, 0.0, scale).astype(np.float32)
    assert xyxy.shape == (batch, k, 4)
    return scores, labels, xyxy

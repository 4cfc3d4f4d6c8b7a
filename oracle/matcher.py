"""CPU oracle for the matching cost and the padded Hungarian solve -- TEST INFRASTRUCTURE.

Restates:

* ``focal_classification_cost`` (``src/rfdetr_jax/models/matcher.py:36-41``);
* ``build_cost_matrix`` for boxes and classes (``matcher.py:44-103,141``): the target class is
  read out of the logits, ``cost = cost_bbox * L1 + cost_class * focal + cost_giou * (-GIoU)``,
  and padded target slots get ``1e4``;
* ``box_cxcywh_to_xyxy`` / ``box_iou`` / ``generalized_box_iou``
  (``src/rfdetr_jax/utilities/box_ops.py:27-75``), keeping the ``1e-7`` clamps;
* ``_solve_batch`` / ``hungarian_match`` (``matcher.py:144-208``): one assignment per
  (image, group) block ``cost[img, g*per_group:(g+1)*per_group, :size]``, non-finite entries
  replaced by ``max(finite) + 1`` (or ``1``), slots ``g*T .. g*T+count`` holding
  ``(row + g*per_group, col, True)`` in ascending row order, unused slots ``(0, 0, False)``.

The solver is SciPy's ``linear_sum_assignment`` -- the reference's own code path -- or the C
restatement in ``oracle/lsap.c``; the two are checked bit-for-bit against each other.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle_lsap.so")
_lib = None

FOCAL_GAMMA = 2.0


def _softplus(x):
    return np.logaddexp(0.0, x)


def focal_classification_cost(logits: np.ndarray, alpha: float) -> np.ndarray:
    """``matcher.py:36-41`` in float64: ``alpha (1-p)^2 softplus(-x) - (1-alpha) p^2 softplus(x)``."""
    x = np.asarray(logits, np.float64)
    prob = 1.0 / (1.0 + np.exp(-x))
    negative = (1 - alpha) * prob ** FOCAL_GAMMA * _softplus(x)  # -log_sigmoid(-x)
    positive = alpha * (1 - prob) ** FOCAL_GAMMA * _softplus(-x)  # -log_sigmoid(x)
    return positive - negative


def box_cxcywh_to_xyxy(boxes: np.ndarray) -> np.ndarray:
    """``box_ops.py:27-32``, negative sizes clamped to zero."""
    cx, cy, w, h = np.moveaxis(np.asarray(boxes, np.float64), -1, 0)
    w = np.clip(w, 0.0, None)
    h = np.clip(h, 0.0, None)
    return np.stack([cx - 0.5 * w, cy - 0.5 * h, cx + 0.5 * w, cy + 0.5 * h], axis=-1)


def generalized_box_iou(boxes1: np.ndarray, boxes2: np.ndarray) -> np.ndarray:
    """Pairwise GIoU for ``[N,4]`` and ``[M,4]`` xyxy boxes (``box_ops.py:46-75``)."""
    area1 = (boxes1[:, 2] - boxes1[:, 0]) * (boxes1[:, 3] - boxes1[:, 1])
    area2 = (boxes2[:, 2] - boxes2[:, 0]) * (boxes2[:, 3] - boxes2[:, 1])
    lt = np.maximum(boxes1[:, None, :2], boxes2[None, :, :2])
    rb = np.minimum(boxes1[:, None, 2:], boxes2[None, :, 2:])
    wh = np.clip(rb - lt, 0.0, None)
    inter = wh[..., 0] * wh[..., 1]
    union = area1[:, None] + area2[None, :] - inter
    iou = inter / np.clip(union, 1e-7, None)
    lt = np.minimum(boxes1[:, None, :2], boxes2[None, :, :2])
    rb = np.maximum(boxes1[:, None, 2:], boxes2[None, :, 2:])
    wh = np.clip(rb - lt, 0.0, None)
    area = wh[..., 0] * wh[..., 1]
    return iou - (area - union) / np.clip(area, 1e-7, None)


def build_cost_matrix(pred_logits, pred_boxes, target_labels, target_boxes, target_mask,
                      cost_class=2.0, cost_bbox=5.0, cost_giou=2.0, focal_alpha=0.25) -> np.ndarray:
    """``[B, Q, T]`` float32 matching cost (``matcher.py:44-103,141``), computed in float64."""
    logits = np.asarray(pred_logits, np.float64)
    boxes = np.asarray(pred_boxes, np.float64)
    labels = np.asarray(target_labels).astype(np.int64)
    tboxes = np.asarray(target_boxes, np.float64)
    mask = np.asarray(target_mask).astype(bool)
    batch, queries, _ = logits.shape
    targets = labels.shape[1]
    cost = np.empty((batch, queries, targets), np.float64)
    for b in range(batch):
        gathered = logits[b][:, labels[b]]  # [Q, T] -- the one-hot einsum of :92-93
        class_cost = focal_classification_cost(gathered, focal_alpha)
        bbox_cost = np.abs(boxes[b][:, None, :] - tboxes[b][None, :, :]).sum(-1)
        giou = generalized_box_iou(box_cxcywh_to_xyxy(boxes[b]), box_cxcywh_to_xyxy(tboxes[b]))
        cost[b] = cost_bbox * bbox_cost + cost_class * class_cost + cost_giou * (-giou)
    cost = np.where(mask[:, None, :], cost, 1e4)
    return cost.astype(np.float32)


def _load_lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            os.makedirs(os.path.dirname(_LIB_PATH), exist_ok=True)
            subprocess.run(["make", "-s", "-C", _HERE], check=True)
        lib = ctypes.CDLL(_LIB_PATH)
        lib.oracle_lsap.restype = ctypes.c_int
        lib.oracle_lsap.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_void_p]
        _lib = lib
    return _lib


def lsap_c(cost: np.ndarray):
    """The C restatement of ``linear_sum_assignment`` (``oracle/lsap.c``); same return as SciPy."""
    cost = np.ascontiguousarray(cost, np.float64)
    if cost.ndim != 2:
        raise ValueError("expected a matrix")
    nr, nc = cost.shape
    count = min(nr, nc)
    rows = np.zeros(count, np.int64)
    cols = np.zeros(count, np.int64)
    status = _load_lib().oracle_lsap(nr, nc, cost.ctypes.data, rows.ctypes.data, cols.ctypes.data)
    if status == -1:
        raise ValueError("matrix contains invalid numeric entries")
    if status != 0:
        raise ValueError("cost matrix is infeasible")
    return rows, cols


def lsap_scipy(cost: np.ndarray):
    """SciPy's solver, the reference's own (``matcher.py:173``)."""
    from scipy.optimize import linear_sum_assignment

    return linear_sum_assignment(cost)


def sanitize_block(block: np.ndarray) -> np.ndarray:
    """``matcher.py:169-172``: replace NaN/+-inf with ``max(finite) + 1`` (float32), or ``1``."""
    if np.isfinite(block).all():
        return block
    finite = block[np.isfinite(block)]
    sentinel = (finite.max() + np.float32(1.0)) if finite.size else np.float32(1.0)
    return np.nan_to_num(block, nan=sentinel, posinf=sentinel, neginf=sentinel)


def solve_batch(cost: np.ndarray, sizes: np.ndarray, group_detr: int, solver=lsap_scipy):
    """``_solve_batch`` (``matcher.py:144-179``) on ``[N, Q, T]`` float32 costs."""
    cost = np.asarray(cost, np.float32)
    batch, num_queries, max_targets = cost.shape
    per_group = num_queries // group_detr
    rows = np.zeros((batch, group_detr * max_targets), np.int32)
    cols = np.zeros((batch, group_detr * max_targets), np.int32)
    valid = np.zeros((batch, group_detr * max_targets), bool)
    for image in range(batch):
        size = int(sizes[image])
        if size == 0:
            continue
        for group in range(group_detr):
            start = group * per_group
            block = sanitize_block(cost[image, start:start + per_group, :size])
            row, col = solver(block)
            offset = group * max_targets
            count = row.shape[0]
            rows[image, offset:offset + count] = row + start
            cols[image, offset:offset + count] = col
            valid[image, offset:offset + count] = True
    return rows, cols, valid


def hungarian_match(cost: np.ndarray, sizes: np.ndarray, group_detr: int, solver=lsap_scipy):
    """``hungarian_match`` (``matcher.py:182-208``): leading axes folded into one batched solve."""
    cost = np.asarray(cost, np.float32)
    leading = cost.shape[:-3]
    batch, _, max_targets = cost.shape[-3:]
    folded = cost.reshape(-1, *cost.shape[-2:])
    folded_sizes = np.broadcast_to(np.asarray(sizes).astype(np.int32), (*leading, batch)).reshape(-1)
    rows, cols, valid = solve_batch(folded, folded_sizes, group_detr, solver)
    shape = (*leading, batch, group_detr * max_targets)
    return rows.reshape(shape), cols.reshape(shape), valid.reshape(shape)

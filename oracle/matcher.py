"""CPU oracle for the matching cost and the padded Hungarian solve -- TEST INFRASTRUCTURE.

Restates:

* ``focal_classification_cost`` (``src/rfdetr_jax/models/matcher.py:36-41``);
* ``build_cost_matrix`` for boxes and classes (``matcher.py:44-103,141``): the target class is
  read out of the logits with the one-hot contraction's semantics (:func:`onehot_gather_f32`),
  in float64 (:func:`build_cost_matrix`) or in float32 in the reference's operation order
  (:func:`build_cost_matrix_f32`), ``cost = cost_bbox * L1 + cost_class * focal + cost_giou * (-GIoU)``,
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
    gathered_all = onehot_gather_f32(logits.astype(np.float32), labels).astype(np.float64)
    for b in range(batch):
        gathered = gathered_all[b]  # [Q, T] -- the one-hot einsum of :92-93 (exact for finite rows)
        class_cost = focal_classification_cost(gathered, focal_alpha)
        bbox_cost = np.abs(boxes[b][:, None, :] - tboxes[b][None, :, :]).sum(-1)
        giou = generalized_box_iou(box_cxcywh_to_xyxy(boxes[b]), box_cxcywh_to_xyxy(tboxes[b]))
        cost[b] = cost_bbox * bbox_cost + cost_class * class_cost + cost_giou * (-giou)
    cost = np.where(mask[:, None, :], cost, 1e4)
    return cost.astype(np.float32)


def onehot_gather_f32(logits: np.ndarray, labels: np.ndarray) -> np.ndarray:
    """``einsum("bqc,btc->bqt", logits, one_hot(labels))`` in float32 (``matcher.py:92-93``).

    For a finite logit row the contraction is exactly ``logits[b, q, label]`` (one product by 1,
    the rest by 0), and 0 for a label outside ``[0, C)`` (``one_hot`` gives an all-zero row).  A
    non-finite logit anywhere else in the row makes its ``x * 0`` term NaN, so the whole row of
    gathered values is NaN -- except an infinite logit at the target's own class with every other
    logit finite, which sums to that infinity.
    """
    logits = np.asarray(logits, np.float32)
    labels = np.asarray(labels).astype(np.int64)
    in_range = (labels >= 0) & (labels < logits.shape[-1])  # an out-of-range label: all-zero one-hot
    safe = np.where(in_range, labels, 0)
    gathered = np.take_along_axis(logits[:, :, None, :], safe[:, None, :, None], -1)[..., 0]
    gathered = np.where(in_range[:, None, :], gathered, np.float32(0))
    bad = ~np.isfinite(logits)  # [B, Q, C]
    n_bad = bad.sum(-1)  # [B, Q]
    own_bad = np.take_along_axis(bad[:, :, None, :], safe[:, None, :, None], -1)[..., 0] & in_range[:, None, :]
    other_bad = (n_bad[:, :, None] - own_bad) > 0
    gathered = np.where(other_bad | np.isnan(gathered), np.float32(np.nan), gathered)
    return gathered.astype(np.float32)


def build_cost_matrix_f32(pred_logits, pred_boxes, target_labels, target_boxes, target_mask,
                          cost_class=2.0, cost_bbox=5.0, cost_giou=2.0, focal_alpha=0.25) -> np.ndarray:
    """``build_cost_matrix`` evaluated in float32 in the reference's operation order.

    Every step rounds to float32 as the reference's ``jnp`` expression does:

    * the one-hot gather of :func:`onehot_gather_f32` (``matcher.py:92-93``);
    * ``focal_classification_cost`` (``matcher.py:36-41``): ``p = sigmoid(x)``,
      ``negative = ((1 - alpha) * p**2) * softplus(x)``, ``positive = (alpha * (1 - p)**2) *
      softplus(-x)`` (``-log_sigmoid(-x)`` is ``softplus(x)``, ``jax.nn.log_sigmoid(x) =
      -softplus(-x)``; ``p**2`` is ``p * p``, the form XLA simplifies ``pow(p, 2)`` to),
      ``positive - negative``;
    * the L1 term ``|pb - tb|`` summed over the four coordinates left to right (``:95``);
    * ``box_cxcywh_to_xyxy`` and ``generalized_box_iou`` (``box_ops.py:27-75``) in float32 with
      the ``1e-7`` clamps;
    * ``cost_bbox * l1 + cost_class * class + cost_giou * (-giou)`` summed left to right
      (``matcher.py:103``), ``1e4`` in padded slots (``:141``).

    ``sigmoid``, ``exp`` and ``log1p`` are NumPy's float32 functions; XLA's may differ in the last
    bit, which is the sensitivity the assignment-flip count measures.
    """
    f = np.float32
    logits = np.asarray(pred_logits, f)
    boxes = np.asarray(pred_boxes, f)
    tboxes = np.asarray(target_boxes, f)
    mask = np.asarray(target_mask).astype(bool)
    with np.errstate(over="ignore", invalid="ignore"):
        x = onehot_gather_f32(logits, target_labels)
        p = (f(1) / (f(1) + np.exp(-x))).astype(f)
        sp_pos = np.logaddexp(x, f(0)).astype(f)
        sp_neg = np.logaddexp(-x, f(0)).astype(f)
        negative = ((f(1 - focal_alpha) * (p * p)) * sp_pos).astype(f)
        q = (f(1) - p).astype(f)
        positive = ((f(focal_alpha) * (q * q)) * sp_neg).astype(f)
        class_cost = (positive - negative).astype(f)
        d = np.abs(boxes[:, :, None, :] - tboxes[:, None, :, :]).astype(f)
        l1 = (((d[..., 0] + d[..., 1]) + d[..., 2]) + d[..., 3]).astype(f)

        def xyxy(bx):
            cx, cy, w, h = bx[..., 0], bx[..., 1], np.clip(bx[..., 2], f(0), None), np.clip(bx[..., 3], f(0), None)
            hw, hh = f(0.5) * w, f(0.5) * h
            return np.stack([cx - hw, cy - hh, cx + hw, cy + hh], -1).astype(f)

        b1 = xyxy(boxes)[:, :, None, :]
        b2 = xyxy(tboxes)[:, None, :, :]
        area1 = ((b1[..., 2] - b1[..., 0]) * (b1[..., 3] - b1[..., 1])).astype(f)
        area2 = ((b2[..., 2] - b2[..., 0]) * (b2[..., 3] - b2[..., 1])).astype(f)
        lt = np.maximum(b1[..., :2], b2[..., :2])
        rb = np.minimum(b1[..., 2:], b2[..., 2:])
        wh = np.clip(rb - lt, f(0), None).astype(f)
        inter = (wh[..., 0] * wh[..., 1]).astype(f)
        union = ((area1 + area2) - inter).astype(f)
        iou = (inter / np.clip(union, f(1e-7), None)).astype(f)
        lt = np.minimum(b1[..., :2], b2[..., :2])
        rb = np.maximum(b1[..., 2:], b2[..., 2:])
        wh = np.clip(rb - lt, f(0), None).astype(f)
        area = (wh[..., 0] * wh[..., 1]).astype(f)
        giou = (iou - ((area - union) / np.clip(area, f(1e-7), None)).astype(f)).astype(f)
        cost = ((f(cost_bbox) * l1 + f(cost_class) * class_cost).astype(f) + f(cost_giou) * (-giou)).astype(f)
    return np.where(mask[:, None, :], cost, f(1e4)).astype(f)


def assignment_objective(cost64: np.ndarray, rows: np.ndarray, cols: np.ndarray, valid: np.ndarray) -> np.ndarray:
    """Total float64 cost of each problem's assignment (``[N, G*T]`` slots of
    :func:`solve_batch`) on ``cost64 [N, Q, T]``."""
    n = cost64.shape[0]
    out = np.zeros(n, np.float64)
    for i in range(n):
        v = valid[i].astype(bool)
        out[i] = cost64[i, rows[i][v], cols[i][v]].sum()
    return out


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

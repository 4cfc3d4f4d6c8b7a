"""CPU oracle for the set-prediction losses of one decoder layer -- test infrastructure only.

Restates, in float64 torch on the host, the reference's matched-pair losses:

* ``loss_labels`` with IA-BCE (``src/rfdetr_jax/models/criterion.py:157-208``): the matched
  (image, query, class) entries get positive weight ``w = clip(p^alpha * iou^(1-alpha), 0.01)``
  (stop-gradient; ``iou`` of the stop-gradient predicted box and the target box,
  ``box_ops.py:78-91``) and negative weight ``1 - w``; every other entry has positive weight 0
  and negative weight ``p^2`` (differentiated); ``loss = sum(neg * x - log_sigmoid(x) * (pos +
  neg)) / num_boxes``;
* ``loss_labels`` without IA-BCE (``criterion.py:210-224``): the sigmoid focal loss (gamma 2) of
  the one-hot matched targets, ``mean(1).sum() / num_boxes`` times the query count;
* ``loss_boxes`` (``criterion.py:233-250``): L1 and ``1 - GIoU`` (``box_ops.py:94-103``) over
  valid matched pairs, each divided by ``num_boxes``.

Gradients come from torch autograd, so they follow the reference's own differentiation of the
same expressions.  The reference's tests pin no values for these losses (they check finiteness
and differentiability only), so this restatement is **parity unpinned**: it follows the code
line by line, and the CUDA kernel is checked against it.
"""

from __future__ import annotations

import numpy as np
import torch


def _xyxy(b):
    cx, cy, w, h = b.unbind(-1)
    w, h = w.clamp(min=0.0), h.clamp(min=0.0)
    return torch.stack([cx - 0.5 * w, cy - 0.5 * h, cx + 0.5 * w, cy + 0.5 * h], -1)


def _iou_union(b1, b2):
    area1 = (b1[..., 2] - b1[..., 0]) * (b1[..., 3] - b1[..., 1])
    area2 = (b2[..., 2] - b2[..., 0]) * (b2[..., 3] - b2[..., 1])
    lt = torch.maximum(b1[..., :2], b2[..., :2])
    rb = torch.minimum(b1[..., 2:], b2[..., 2:])
    wh = (rb - lt).clamp(min=0.0)
    inter = wh[..., 0] * wh[..., 1]
    union = area1 + area2 - inter
    return inter / union.clamp(min=1e-7), union


def _giou(b1, b2):
    iou, union = _iou_union(b1, b2)
    lt = torch.minimum(b1[..., :2], b2[..., :2])
    rb = torch.maximum(b1[..., 2:], b2[..., 2:])
    wh = (rb - lt).clamp(min=0.0)
    area = wh[..., 0] * wh[..., 1]
    return iou - (area - union) / area.clamp(min=1e-7)


def set_losses(pred_logits, pred_boxes, target_labels, target_boxes, rows, cols, valid, num_boxes,
               focal_alpha=0.25, ia_bce=True):
    """``(loss_ce, loss_bbox, loss_giou)`` and their gradients with respect to the logits and the
    boxes (for unit cotangents), all float64 numpy.

    Args:
        pred_logits ``[B, Q, C]``, pred_boxes ``[B, Q, 4]`` (cxcywh); target_labels ``[B, T]``,
        target_boxes ``[B, T, 4]``; rows/cols/valid ``[B, S]`` from the matcher; num_boxes the
        loss denominator.
    """
    x = torch.tensor(np.asarray(pred_logits, np.float64), requires_grad=True)
    pb = torch.tensor(np.asarray(pred_boxes, np.float64), requires_grad=True)
    labels = torch.tensor(np.asarray(target_labels, np.int64))
    tboxes = torch.tensor(np.asarray(target_boxes, np.float64))
    rows = torch.tensor(np.asarray(rows, np.int64))
    cols = torch.tensor(np.asarray(cols, np.int64))
    valid = torch.tensor(np.asarray(valid, bool))
    batch, queries, classes = x.shape
    bidx = torch.arange(batch)[:, None].expand_as(rows)
    rclip = rows.clamp(0, queries - 1)
    tcls = torch.gather(labels, 1, cols)                                   # criterion.py:184
    tgt = torch.gather(tboxes, 1, cols[..., None].expand(-1, -1, 4))

    if ia_bce:
        loss_ce = _ia_bce(x, pb, tgt, tcls, bidx, rows, rclip, valid, num_boxes, focal_alpha)
    else:
        loss_ce = _focal(x, tcls, bidx, rows, valid, num_boxes, focal_alpha)

    # loss_boxes (criterion.py:233-250).
    srcb = pb[bidx, rclip]
    w = valid.to(torch.float64)
    l1 = ((srcb - tgt).abs().sum(-1) * w).sum() / num_boxes
    giou = ((1 - _giou(_xyxy(srcb), _xyxy(tgt))) * w).sum() / num_boxes

    (g_ce,) = torch.autograd.grad(loss_ce, x, retain_graph=True)
    (g_l1,) = torch.autograd.grad(l1, pb, retain_graph=True)
    (g_giou,) = torch.autograd.grad(giou, pb)
    return (float(loss_ce.detach()), float(l1.detach()), float(giou.detach()), g_ce.numpy(), g_l1.numpy(),
            g_giou.numpy())


def _ia_bce(x, pb, tgt, tcls, bidx, rows, rclip, valid, num_boxes, focal_alpha):
    """loss_labels, IA-BCE (criterion.py:188-208)."""
    src = pb[bidx, rclip].detach()
    iou, _ = _iou_union(_xyxy(src), _xyxy(tgt))
    prob = torch.sigmoid(x)
    matched_prob = prob[bidx, rclip, tcls]
    weight = (matched_prob.pow(focal_alpha) * iou.pow(1 - focal_alpha)).detach().clamp(min=0.01)
    weight = torch.where(valid, weight, torch.zeros_like(weight))
    pos = torch.zeros_like(x)
    neg = prob.pow(2.0)
    sel = valid
    pos = pos.index_put((bidx[sel], rows[sel], tcls[sel]), weight[sel])
    neg = neg.index_put((bidx[sel], rows[sel], tcls[sel]), 1 - weight[sel])
    return (neg * x - torch.nn.functional.logsigmoid(x) * (pos + neg)).sum() / num_boxes


def _focal(x, tcls, bidx, rows, valid, num_boxes, alpha, gamma=2.0):
    """loss_labels without IA-BCE (criterion.py:210-224): sigmoid focal loss of the one-hot matched
    targets, ``mean(1).sum() / num_boxes`` times the query count."""
    sel = valid
    onehot = torch.zeros_like(x).index_put((bidx[sel], rows[sel], tcls[sel]), torch.ones(int(sel.sum()),
                                                                                        dtype=x.dtype))
    prob = torch.sigmoid(x)
    ce = torch.nn.functional.binary_cross_entropy_with_logits(x, onehot, reduction="none")
    p_t = prob * onehot + (1 - prob) * (1 - onehot)
    loss = ce * (1 - p_t) ** gamma
    if alpha >= 0:
        loss = (alpha * onehot + (1 - alpha) * (1 - onehot)) * loss
    return loss.mean(1).sum() / num_boxes * x.shape[1]

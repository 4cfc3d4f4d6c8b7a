"""Set-prediction losses on B200 (IA-BCE or focal classification, L1 and GIoU box terms over
matched pairs), mirroring ``loss_labels`` / ``loss_boxes`` of
``src/rfdetr_jax/models/criterion.py:157-250``.

One library launch computes the three losses of every stacked layer and their gradients with
respect to the logits and the boxes; :class:`SetLossFunction` returns the losses and, in
backward, scales the stored gradients by the incoming cotangents (the IA-BCE weights are
stop-gradient in the reference, so the classification loss has no box gradient).
"""

from __future__ import annotations

import math

import torch

from . import _native as N


class SetLossFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pred_logits, pred_boxes, target_labels, target_boxes, rows, cols, valid, num_boxes, focal_alpha,
                ia_bce):
        N.require_cuda(pred_logits, pred_boxes, target_labels, target_boxes, rows, cols, valid)
        if pred_logits.dim() < 3:
            raise ValueError("pred_logits must be [..., B, Q, C]")
        leading = pred_logits.shape[:-3]
        batch, queries, classes = pred_logits.shape[-3:]
        layers = math.prod(leading)
        targets = target_labels.shape[-1]
        slots = rows.shape[-1]
        if pred_boxes.shape != (*leading, batch, queries, 4) or target_labels.shape != (batch, targets) \
                or target_boxes.shape != (batch, targets, 4) or rows.shape != (*leading, batch, slots) \
                or cols.shape != rows.shape or valid.shape != rows.shape:
            raise ValueError("inconsistent shapes for set_losses")
        dev = pred_logits.device
        logits = pred_logits.detach().to(torch.float32).contiguous()
        boxes = pred_boxes.detach().to(torch.float32).contiguous()
        nb = (num_boxes if torch.is_tensor(num_boxes) else torch.tensor(float(num_boxes)))
        nb = nb.to(device=dev, dtype=torch.float32).reshape(1).contiguous()
        losses = torch.empty((*leading, 3), dtype=torch.float32, device=dev)
        g_logits = torch.empty_like(logits)
        g_l1 = torch.empty_like(boxes)
        g_giou = torch.empty_like(boxes)
        status = N.lib().rfdetr_set_losses(
            N.stream_of(logits), N.ptr(logits), N.ptr(boxes), N.ptr(target_labels.to(torch.int32).contiguous()),
            N.ptr(target_boxes.to(torch.float32).contiguous()), N.ptr(rows.to(torch.int32).contiguous()),
            N.ptr(cols.to(torch.int32).contiguous()), N.ptr(valid.to(torch.uint8).contiguous()), N.ptr(nb), layers,
            batch, queries, classes, targets, slots, float(focal_alpha), int(bool(ia_bce)), N.ptr(losses),
            N.ptr(g_logits), N.ptr(g_l1), N.ptr(g_giou))
        N.check(status, "rfdetr_set_losses")
        ctx.save_for_backward(g_logits, g_l1, g_giou)
        ctx.dtypes = (pred_logits.dtype, pred_boxes.dtype)
        return losses[..., 0], losses[..., 1], losses[..., 2]

    @staticmethod
    def backward(ctx, g_ce, g_bbox, g_giou):
        g_logits, g_l1, g_gi = ctx.saved_tensors
        per = lambda g: g[..., None, None, None]  # noqa: E731  (a cotangent per layer)
        d_logits = (g_logits * per(g_ce)).to(ctx.dtypes[0])
        d_boxes = (g_l1 * per(g_bbox) + g_gi * per(g_giou)).to(ctx.dtypes[1])
        return d_logits, d_boxes, None, None, None, None, None, None, None, None


def set_losses(pred_logits, pred_boxes, target_labels, target_boxes, rows, cols, valid, num_boxes, focal_alpha=0.25,
               ia_bce=True):
    """``(loss_ce, loss_bbox, loss_giou)``: ``loss_labels`` (``criterion.py:157-224``; IA-BCE when
    ``ia_bce``, else the sigmoid focal loss with gamma 2) and the matched-pair box losses
    (``criterion.py:233-250``), differentiable with respect to ``pred_logits`` and ``pred_boxes``.

    ``pred_logits [..., B, Q, C]`` and ``pred_boxes [..., B, Q, 4]`` may carry leading layer axes
    (all layers in one launch); ``rows/cols/valid [..., B, S]`` are the matcher's outputs for the
    same layers (``hungarian_match`` of the stacked costs); targets ``[B, T]`` / ``[B, T, 4]`` are
    shared.  Each loss has the leading shape (a scalar for one layer)."""
    return SetLossFunction.apply(pred_logits, pred_boxes, target_labels, target_boxes, rows, cols, valid, num_boxes,
                                 focal_alpha, ia_bce)

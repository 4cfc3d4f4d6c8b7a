"""Inference post-process on B200: the top-k over all query/class pairs.

Mirrors ``src/rfdetr_jax/models/postprocess.py:19-51`` (``post_process``): sigmoid scores of
``[B, Q, C]`` logits flattened to ``[B, Q*C]``, ``jax.lax.top_k`` of ``num_select`` of them
(here the library's radix select, bit-exact with ``lax.top_k``: descending, lower flattened index
first on ties, NaN first), query = index // C, label = index % C, and the selected boxes
converted to absolute ``xyxy`` clamped to the image (``box_ops.py:27-32``).  The sigmoid and the
box arithmetic are elementwise device ops around the selection.
"""

from __future__ import annotations

import torch

from . import _native as N
from .topk import top_k


def post_process(pred_logits: torch.Tensor, pred_boxes: torch.Tensor, target_sizes: torch.Tensor,
                 num_select: int = 300):
    """``(scores [B, K], labels int32 [B, K], boxes [B, K, 4])`` as the reference's ``post_process``.

    Args:
        pred_logits: ``[B, Q, C]`` classification logits (float32, or cast to it).
        pred_boxes: ``[B, Q, 4]`` normalized ``cxcywh`` boxes.
        target_sizes: ``[B, 2]`` per-image ``(height, width)``.
        num_select: detections per image; ``K = min(num_select, Q * C)``.
    """
    N.require_cuda(pred_logits, pred_boxes, target_sizes)
    batch, queries, classes = pred_logits.shape
    if pred_boxes.shape != (batch, queries, 4) or target_sizes.shape != (batch, 2):
        raise ValueError("inconsistent shapes for post_process")
    probabilities = torch.sigmoid(pred_logits.to(torch.float32)).reshape(batch, -1)
    k = min(int(num_select), probabilities.shape[1])
    scores, indexes = top_k(probabilities, k)
    query_index = torch.div(indexes, classes, rounding_mode="floor")
    labels = (indexes - query_index * classes).to(torch.int32)
    boxes = pred_boxes.to(torch.float32)
    cx, cy, w, h = boxes.unbind(-1)
    w, h = w.clamp(min=0.0), h.clamp(min=0.0)
    xyxy = torch.stack([cx - 0.5 * w, cy - 0.5 * h, cx + 0.5 * w, cy + 0.5 * h], dim=-1)
    xyxy = torch.gather(xyxy, 1, query_index.to(torch.int64)[..., None].expand(-1, -1, 4))
    height = target_sizes[:, 0].to(xyxy.dtype)
    width = target_sizes[:, 1].to(xyxy.dtype)
    scale = torch.stack([width, height, width, height], dim=1)[:, None, :]
    xyxy = torch.minimum(torch.clamp(xyxy * scale, min=0.0), scale)
    return scores, labels, xyxy

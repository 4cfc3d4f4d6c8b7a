"""Matching cost and exact batched assignment on B200.

Mirrors ``src/rfdetr_jax/models/matcher.py`` and the solver switch of
``src/rfdetr_jax/models/criterion.py:79-90``:

* :func:`build_cost_matrix` -- the class/L1/GIoU cost with ``1e4`` on padded targets
  (``matcher.py:44-103,141``);
* :func:`hungarian_match` -- ``(cost [..., B, Q, T], sizes [B], group_detr) -> (rows, cols,
  valid)`` each ``[..., B, group_detr * T]`` (``matcher.py:182-208``), solved on the device with
  SciPy's algorithm and tie rules, so the assignment equals the reference's host solve;
* :func:`match_stacked` -- cost and assignment of all stacked layers in one call
  (``criterion.py:402-413``: the stacked ``layer_cost`` then one ``solve``);
* :class:`CriterionConfig` -- ``solve`` dispatch with ``matcher="cuda"``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native as N
from ._native import check_device_status  # noqa: F401  (re-exported)


def build_cost_matrix(pred_logits: torch.Tensor, pred_boxes: torch.Tensor, target_labels: torch.Tensor,
                      target_boxes: torch.Tensor, target_mask: torch.Tensor, cost_class: float, cost_bbox: float,
                      cost_giou: float, focal_alpha: float, **unsupported) -> torch.Tensor:
    """``[B, Q, T]`` float32 matching cost (reference ``matcher.py:44-141``, boxes and classes).

    Keypoint and mask cost terms (``matcher.py:105-138``) are not part of this backend; passing
    them raises ``NotImplementedError``.
    """
    extra = {k: v for k, v in unsupported.items() if v is not None and v != () and v != (0.0, 0.0)
             and v != (0.0, 0.0, 0.0, 0.0)}
    if extra:
        raise NotImplementedError(f"cost terms not implemented by the cuda backend: {sorted(extra)}")
    N.require_cuda(pred_logits, pred_boxes, target_labels, target_boxes, target_mask)
    batch, queries, classes = pred_logits.shape
    targets = target_labels.shape[1]
    if pred_boxes.shape != (batch, queries, 4) or target_boxes.shape != (batch, targets, 4) \
            or target_mask.shape != (batch, targets):
        raise ValueError("inconsistent shapes for build_cost_matrix")
    cost = torch.empty((batch, queries, targets), dtype=torch.float32, device=pred_logits.device)
    logits = pred_logits.contiguous()
    boxes = pred_boxes.contiguous()
    labels = target_labels.to(torch.int32).contiguous()
    tboxes = target_boxes.to(torch.float32).contiguous()
    mask = target_mask.to(torch.uint8).contiguous()
    status = N.lib().rfdetr_match_cost(
        N.stream_of(logits), N.ptr(logits), N.dtype_code(logits.dtype), N.ptr(boxes), N.dtype_code(boxes.dtype),
        N.ptr(labels), N.ptr(tboxes), N.ptr(mask), N.ptr(cost), batch, queries, classes, targets,
        float(cost_class), float(cost_bbox), float(cost_giou), float(focal_alpha))
    N.check(status, "rfdetr_match_cost")
    return cost


def match_stacked(pred_logits: torch.Tensor, pred_boxes: torch.Tensor, target_labels: torch.Tensor,
                  target_boxes: torch.Tensor, target_mask: torch.Tensor, sizes: torch.Tensor, group_detr: int,
                  cost_class: float, cost_bbox: float, cost_giou: float, focal_alpha: float, check: bool = False,
                  status: torch.Tensor | None = None):
    """Cost and exact assignment of every stacked layer in one call: one cost launch over all
    layers and images, then one batched solve (bit for bit :func:`build_cost_matrix` per layer
    followed by :func:`hungarian_match` of the stacked cost).

    Args:
        pred_logits ``[..., B, Q, C]``, pred_boxes ``[..., B, Q, 4]`` (leading axes: layers);
        target_labels ``[B, T]``, target_boxes ``[B, T, 4]``, target_mask ``[B, T]`` shared by the
        layers; sizes ``[B]``; group_detr divides ``Q``.

        check: read the device status word right away (synchronises the stream).  Off by
            default: the status only reports a solve that reached its iteration cap, which finite
            costs never do, and reading it every step would stall the stream.
        status: optional device ``int32`` tensor (one element, zero before the first call) that
            receives the status; it is only ever raised, so one tensor can collect many calls and
            be read once with :func:`check_device_status`.

    Returns:
        ``(cost [..., B, Q, T] float32, rows int32, cols int32, valid bool)``, the last three
        ``[..., B, group_detr * T]``.
    """
    N.require_cuda(pred_logits, pred_boxes, target_labels, target_boxes, target_mask, sizes)
    if pred_logits.dim() < 3:
        raise ValueError("pred_logits must be [..., B, Q, C]")
    leading = pred_logits.shape[:-3]
    batch, queries, classes = pred_logits.shape[-3:]
    targets = target_labels.shape[-1]
    if pred_boxes.shape != (*leading, batch, queries, 4) or target_labels.shape != (batch, targets) \
            or target_boxes.shape != (batch, targets, 4) or target_mask.shape != (batch, targets) \
            or sizes.shape != (batch,):
        raise ValueError("inconsistent shapes for match_stacked")
    if group_detr < 1 or queries % group_detr:
        raise ValueError("group_detr must be positive and divide the query count")
    layers = 1
    for d in leading:
        layers *= d
    dev = pred_logits.device
    logits = pred_logits.contiguous()
    boxes = pred_boxes.contiguous()
    slots = group_detr * targets
    cost = torch.empty((*leading, batch, queries, targets), dtype=torch.float32, device=dev)
    rows = torch.empty((*leading, batch, slots), dtype=torch.int32, device=dev)
    cols = torch.empty_like(rows)
    valid = torch.empty((*leading, batch, slots), dtype=torch.uint8, device=dev)
    status_buf = _status_buffer(status, dev)
    st = N.lib().rfdetr_match_stacked(
        N.stream_of(logits), N.ptr(logits), N.dtype_code(logits.dtype), N.ptr(boxes), N.dtype_code(boxes.dtype),
        N.ptr(target_labels.to(torch.int32).contiguous()), N.ptr(target_boxes.to(torch.float32).contiguous()),
        N.ptr(target_mask.to(torch.uint8).contiguous()), N.ptr(sizes.to(torch.int32).contiguous()), layers, batch,
        queries, classes, targets, group_detr, float(cost_class), float(cost_bbox), float(cost_giou),
        float(focal_alpha), N.ptr(cost), N.ptr(rows), N.ptr(cols), N.ptr(valid), N.ptr(status_buf))
    N.check(st, "rfdetr_match_stacked")
    if check:
        N.check_device_status(status_buf, "rfdetr_match_stacked (device status)")
    return cost, rows, cols, valid.to(torch.bool)


def _status_buffer(status, device):
    if status is None:
        return torch.zeros((1,), dtype=torch.int32, device=device)
    if status.dtype != torch.int32 or status.numel() < 1 or status.device != device or not status.is_contiguous():
        raise ValueError("status must be a contiguous int32 tensor on the cost's device")
    return status


def hungarian_match(cost: torch.Tensor, sizes: torch.Tensor, group_detr: int, check: bool = False,
                    status: torch.Tensor | None = None):
    """Exact assignment of every (layer, image, group) block in one launch.

    Args:
        cost: ``[..., B, Q, T]``; cast to float32 as the reference does (``matcher.py:203``).
        sizes: real target count per image ``[B]``.
        group_detr: number of query groups; must divide ``Q``.
        check: read the device status word right away (synchronises the stream).  Off by
            default: a solve only reports a status when it reaches its iteration cap, which
            finite costs never do, and reading it every step would stall the stream.
        status: optional device ``int32`` tensor (one element, zero before the first call) that
            receives ``RFDETR_ERR_LIMIT`` if a solve gives up; the word is only ever raised, so one
            tensor can collect many calls and be read once with :func:`check_device_status`.
            A block whose solve gives up keeps its cleared slots ``(0, 0, False)``.

    Returns:
        ``(rows int32, cols int32, valid bool)``, each ``[..., B, group_detr * T]``.
    """
    N.require_cuda(cost, sizes)
    leading = cost.shape[:-3]
    batch, queries, max_targets = cost.shape[-3:]
    if group_detr < 1 or queries % group_detr:
        raise ValueError("group_detr must be positive and divide the query count")
    folded = cost.detach().to(torch.float32).reshape(-1, queries, max_targets).contiguous()
    folded_sizes = torch.broadcast_to(sizes.to(torch.int32), (*leading, batch)).reshape(-1).contiguous()
    problems = folded.shape[0]
    slots = group_detr * max_targets
    rows = torch.empty((problems, slots), dtype=torch.int32, device=cost.device)
    cols = torch.empty((problems, slots), dtype=torch.int32, device=cost.device)
    valid = torch.empty((problems, slots), dtype=torch.uint8, device=cost.device)
    status_buf = _status_buffer(status, cost.device)
    st = N.lib().rfdetr_lsap_batched(N.stream_of(folded), N.ptr(folded), N.ptr(folded_sizes), problems, queries,
                                     max_targets, group_detr, N.ptr(rows), N.ptr(cols), N.ptr(valid),
                                     N.ptr(status_buf))
    N.check(st, "rfdetr_lsap_batched")
    if check:
        N.check_device_status(status_buf, "rfdetr_lsap_batched (device status)")
    shape = (*leading, batch, slots)
    return rows.reshape(shape), cols.reshape(shape), valid.to(torch.bool).reshape(shape)


MATCHERS = ("cuda", "hungarian")


@dataclass(frozen=True)
class CriterionConfig:
    """The solver switch of the reference's ``CriterionConfig`` (``criterion.py:37-90``).

    ``matcher="cuda"`` (and ``"hungarian"``, the reference's exact matcher, which here runs on the
    device with identical results) solve exactly on the GPU inside the step: no host round trip,
    so it also works per shard under data parallelism.
    """

    focal_alpha: float = 0.25
    group_detr: int = 13
    set_cost_class: float = 2.0
    set_cost_bbox: float = 5.0
    set_cost_giou: float = 2.0
    matcher: str = "cuda"

    def solve(self, cost: torch.Tensor, sizes: torch.Tensor, group_detr: int):
        if self.matcher in MATCHERS:
            return hungarian_match(cost, sizes, group_detr)
        raise ValueError(f"unknown matcher {self.matcher!r}; expected 'cuda' or 'hungarian'")

    def cost(self, pred_logits, pred_boxes, target_labels, target_boxes, target_mask):
        return build_cost_matrix(pred_logits, pred_boxes, target_labels, target_boxes, target_mask,
                                 self.set_cost_class, self.set_cost_bbox, self.set_cost_giou, self.focal_alpha)

    def match(self, pred_logits, pred_boxes, target_labels, target_boxes, target_mask, sizes, group_detr):
        """The stacked ``layer_cost`` + ``solve`` of ``compute_losses`` (``criterion.py:402-413``)
        in one call; returns ``(rows, cols, valid)``."""
        if self.matcher not in MATCHERS:
            raise ValueError(f"unknown matcher {self.matcher!r}; expected 'cuda' or 'hungarian'")
        _, rows, cols, valid = match_stacked(pred_logits, pred_boxes, target_labels, target_boxes, target_mask,
                                             sizes, group_detr, self.set_cost_class, self.set_cost_bbox,
                                             self.set_cost_giou, self.focal_alpha)
        return rows, cols, valid

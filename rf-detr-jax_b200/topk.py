"""Two-stage query selection on B200.

Mirrors ``src/rfdetr_jax/models/transformer.py:694-706`` and ``layers.py:225-244``:

* :func:`two_stage_topk` -- ``proposal_scores = logits.max(-1)`` then
  ``jax.lax.top_k(proposal_scores, k)`` fused in one launch;
* :func:`top_k` -- ``jax.lax.top_k`` over the last axis (descending, lower index first on ties,
  IEEE totalOrder with NaN first);
* :func:`select_rows` -- the batched row gather that follows the selection.
"""

from __future__ import annotations

import torch

from . import _native as N


def _topk(logits: torch.Tensor, k: int, want_scores: bool):
    N.require_cuda(logits)
    if logits.dtype != torch.float32:
        raise ValueError("the selection kernel takes float32 scores/logits")
    *lead, positions, classes = logits.shape
    if not 1 <= k <= positions:
        raise ValueError(f"k={k} must be in [1, {positions}]")
    rows = 1
    for d in lead:
        rows *= d
    logits = logits.contiguous()
    scores = torch.empty((*lead, positions), dtype=torch.float32, device=logits.device) if want_scores else None
    values = torch.empty((*lead, k), dtype=torch.float32, device=logits.device)
    indices = torch.empty((*lead, k), dtype=torch.int32, device=logits.device)
    status = N.lib().rfdetr_topk_select(N.stream_of(logits), N.ptr(logits), rows, positions, classes, k,
                                        N.ptr(scores), N.ptr(values), N.ptr(indices))
    N.check(status, "rfdetr_topk_select")
    return scores, values, indices


def two_stage_topk(logits: torch.Tensor, num_queries: int):
    """Class max + top-k over proposals (``transformer.py:694-696``).

    Args:
        logits: ``[..., positions, classes]`` float32.
        num_queries: selection size; ``k = min(num_queries, positions)`` (``transformer.py:694``).

    Returns:
        ``(proposal_scores [..., positions], topk_values [..., k], topk_indices int32 [..., k])``.
    """
    k = min(int(num_queries), logits.shape[-2])
    return _topk(logits, k, True)


def top_k(scores: torch.Tensor, k: int):
    """``jax.lax.top_k(scores, k)`` over the last axis: ``(values, int32 indices)``."""
    _, values, indices = _topk(scores.unsqueeze(-1), int(k), False)
    return values, indices


def select_rows(values: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    """Gather rows of ``values [..., N, C]`` at ``indices [..., K]`` (``layers.py:225-244``).

    Indices must be in bounds (the reference uses ``mode="promise_in_bounds"``); an
    out-of-range index raises ``ValueError`` here (checked after the launch).
    """
    N.require_cuda(values, indices)
    lead = indices.shape[:-1]
    if values.shape[:-2] != lead:
        raise ValueError("values and indices must share their leading axes")
    k = indices.shape[-1]
    positions, width = values.shape[-2], values.shape[-1]
    rows = 1
    for d in lead:
        rows *= d
    values = values.contiguous()
    idx = indices.to(torch.int32).contiguous()
    out = torch.empty((*lead, k, width), dtype=values.dtype, device=values.device)
    status_buf = torch.zeros((1,), dtype=torch.int32, device=values.device)
    status = N.lib().rfdetr_select_rows(N.stream_of(values), N.ptr(values), values.element_size(), rows, positions,
                                        width, N.ptr(idx), k, N.ptr(out), N.ptr(status_buf))
    N.check(status, "rfdetr_select_rows")
    code = int(status_buf.item())
    if code:
        raise ValueError("select_rows: an index is out of bounds")
    return out

"""Multi-scale deformable attention on B200: the ``"cuda"`` sampler.

Mirrors the reference's operator interface (``src/rfdetr_jax/models/ops.py``):

* :func:`ms_deform_attn_core_rows` -- same arguments as the reference (``ops.py:208-292``),
  channels-last ``value [B*H, sum(HW), D]``; ``sampler`` must be ``"cuda"`` and any other name is
  rejected with the reference's ``ValueError("unknown sampler ...")`` (``ops.py:235-238``);
* :func:`ms_deform_attn_core` -- the ``[B, H, D, sum(HW)]`` entry point (``ops.py:295-314``);
* :func:`ms_deform_attn` -- the signature of the drop-in contract,
  ``(value, spatial_shapes, level_start_index, sampling_locations, attention_weights)``.

Autodiff mirrors the reference's ``custom_vjp`` pattern (``deform_pallas.py:132-178``): a
``torch.autograd.Function`` whose backward returns ``(grad_value, grad_locations,
grad_weights)`` in the input dtypes.  Output dtype is ``result_type(value, weights)``
(``ops.py:260``).  Sampling locations are used in float32 (the reference promotes to at least
float32, ``ops.py:270``); float64 locations are rejected rather than silently narrowed.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch

from . import _native as N

SAMPLERS = ("cuda",)


def _shapes_tuple(spatial_shapes) -> tuple[tuple[int, int], ...]:
    if isinstance(spatial_shapes, torch.Tensor):
        spatial_shapes = spatial_shapes.tolist()
    return tuple((int(h), int(w)) for h, w in spatial_shapes)


def _prepare(value, spatial_shapes, sampling_locations, attention_weights):
    shapes = _shapes_tuple(spatial_shapes)
    N.require_cuda(value, sampling_locations, attention_weights)
    if sampling_locations.dim() != 6 or sampling_locations.shape[-1] != 2:
        raise ValueError("sampling_locations must be [B, Lq, n_heads, n_levels, n_points, 2]")
    batch, len_query, heads, levels, points, _ = sampling_locations.shape
    if len(shapes) != levels:
        raise ValueError(f"spatial_shapes has {len(shapes)} levels but sampling_locations has {levels}")
    total = sum(h * w for h, w in shapes)
    if value.dim() != 3 or value.shape[0] != batch * heads or value.shape[1] != total:
        raise ValueError(f"value must be [B * n_heads, sum(H*W), head_dim] = [{batch * heads}, {total}, D], "
                         f"got {list(value.shape)}")
    if tuple(attention_weights.shape) != (batch, len_query, heads, levels * points):
        raise ValueError("attention_weights must be [B, Lq, n_heads, n_levels * n_points]")
    if sampling_locations.dtype == torch.float64:
        raise ValueError("float64 sampling_locations are not supported by the cuda sampler")
    if sampling_locations.dtype != torch.float32:
        sampling_locations = sampling_locations.float()  # exact widening, as ops.py:270 promotes
    value = value.contiguous()
    sampling_locations = sampling_locations.contiguous()
    attention_weights = attention_weights.contiguous()
    return shapes, value, sampling_locations, attention_weights


def _out_dtype(value_dtype, weight_dtype):
    return torch.bfloat16 if (value_dtype == torch.bfloat16 and weight_dtype == torch.bfloat16) else torch.float32


def msda_forward(value, shapes, sampling_locations, attention_weights) -> torch.Tensor:
    """One forward launch; inputs already validated and contiguous."""
    batch, len_query, heads, levels, points, _ = sampling_locations.shape
    dim = value.shape[-1]
    out = torch.empty((batch, len_query, heads * dim), dtype=_out_dtype(value.dtype, attention_weights.dtype),
                      device=value.device)
    flat = [v for hw in shapes for v in hw]
    status = N.lib().rfdetr_msda_forward(
        N.stream_of(value), N.ptr(value), N.dtype_code(value.dtype), N.int64_array(flat), None,
        N.ptr(sampling_locations), N.ptr(attention_weights), N.dtype_code(attention_weights.dtype),
        N.ptr(out), N.dtype_code(out.dtype), batch, heads, dim, len_query, levels, points)
    N.check(status, "rfdetr_msda_forward")
    return out


def msda_backward(value, shapes, sampling_locations, attention_weights, grad_output):
    """One backward launch; returns ``(grad_value, grad_locations, grad_weights)``."""
    batch, len_query, heads, levels, points, _ = sampling_locations.shape
    dim = value.shape[-1]
    expected = _out_dtype(value.dtype, attention_weights.dtype)
    grad_output = grad_output.to(expected).contiguous()
    grad_value = torch.empty_like(value)
    grad_loc = torch.empty_like(sampling_locations)
    grad_attn = torch.empty_like(attention_weights)
    lib = N.lib()
    ws_bytes = lib.rfdetr_msda_backward_workspace_size(N.dtype_code(value.dtype), batch, heads, dim, value.shape[1])
    workspace = torch.empty(max(int(ws_bytes), 1), dtype=torch.uint8, device=value.device) if ws_bytes else None
    flat = [v for hw in shapes for v in hw]
    status = lib.rfdetr_msda_backward(
        N.stream_of(value), N.ptr(value), N.dtype_code(value.dtype), N.int64_array(flat), None,
        N.ptr(sampling_locations), N.ptr(attention_weights), N.dtype_code(attention_weights.dtype),
        N.ptr(grad_output), N.dtype_code(grad_output.dtype), N.ptr(grad_value), N.ptr(grad_loc),
        N.ptr(grad_attn), N.ptr(workspace), int(ws_bytes), batch, heads, dim, len_query, levels, points)
    N.check(status, "rfdetr_msda_backward")
    return grad_value, grad_loc, grad_attn


class MSDeformAttnFunction(torch.autograd.Function):
    """Sampler forward with the analytic CUDA backward (the reference's custom_vjp pattern)."""

    @staticmethod
    def forward(ctx, value, sampling_locations, attention_weights, shapes):
        out = msda_forward(value, shapes, sampling_locations, attention_weights)
        ctx.save_for_backward(value, sampling_locations, attention_weights)
        ctx.shapes = shapes
        return out

    @staticmethod
    def backward(ctx, grad_output):
        value, sampling_locations, attention_weights = ctx.saved_tensors
        grad_value, grad_loc, grad_attn = msda_backward(value, ctx.shapes, sampling_locations, attention_weights,
                                                        grad_output)
        return (grad_value if ctx.needs_input_grad[0] else None,
                grad_loc if ctx.needs_input_grad[1] else None,
                grad_attn if ctx.needs_input_grad[2] else None,
                None)


def ms_deform_attn_core_rows(value: torch.Tensor, spatial_shapes: Sequence[Sequence[int]],
                             sampling_locations: torch.Tensor, attention_weights: torch.Tensor,
                             sampler: str = "cuda") -> torch.Tensor:
    """Sample and weight multi-scale features, channels last (reference ``ops.py:208-292``).

    Args:
        value: ``[B * n_heads, sum(H*W), head_dim]`` float32 or bfloat16.
        spatial_shapes: per-level ``(H, W)``.
        sampling_locations: ``[B, Lq, n_heads, n_levels, n_points, 2]`` in ``[0, 1]``.
        attention_weights: ``[B, Lq, n_heads, n_levels * n_points]``.
        sampler: ``"cuda"``.

    Returns:
        ``[B, Lq, n_heads * head_dim]`` in ``result_type(value, attention_weights)``.
    """
    if sampler not in SAMPLERS:
        raise ValueError(f"unknown sampler {sampler!r}; expected 'cuda'")
    shapes, value, sampling_locations, attention_weights = _prepare(
        value, spatial_shapes, sampling_locations, attention_weights)
    if sampling_locations.shape[1] == 0:
        b, _, h, _, _, _ = sampling_locations.shape
        return value.new_zeros((b, 0, h * value.shape[-1]), dtype=_out_dtype(value.dtype, attention_weights.dtype))
    return MSDeformAttnFunction.apply(value, sampling_locations, attention_weights, shapes)


def ms_deform_attn_core(value: torch.Tensor, spatial_shapes, sampling_locations, attention_weights,
                        sampler: str = "cuda") -> torch.Tensor:
    """``[B, n_heads, head_dim, sum(H*W)]`` entry point (reference ``ops.py:295-314``)."""
    batch, heads, dim, length = value.shape
    rows = value.permute(0, 1, 3, 2).reshape(batch * heads, length, dim)
    return ms_deform_attn_core_rows(rows, spatial_shapes, sampling_locations, attention_weights, sampler)


def ms_deform_attn(value: torch.Tensor, spatial_shapes, level_start_index, sampling_locations: torch.Tensor,
                   attention_weights: torch.Tensor) -> torch.Tensor:
    """The drop-in signature ``(value, spatial_shapes, level_start_index, sampling_locations,
    attention_weights)``.  ``level_start_index`` must match the cumulative level sizes (the
    reference derives it from ``spatial_shapes``, ``ops.py:265-267``)."""
    shapes = _shapes_tuple(spatial_shapes)
    if level_start_index is not None:
        starts = [int(s) for s in (level_start_index.tolist() if isinstance(level_start_index, torch.Tensor)
                                   else level_start_index)]
        expected, total = [], 0
        for h, w in shapes:
            expected.append(total)
            total += h * w
        if starts != expected:
            raise ValueError(f"level_start_index {starts} does not match spatial_shapes (expected {expected})")
    return ms_deform_attn_core_rows(value, shapes, sampling_locations, attention_weights, "cuda")

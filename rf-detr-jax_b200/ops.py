"""Multi-scale deformable attention on B200: the ``"cuda"`` sampler.

Mirrors the reference's operator interface (``src/rfdetr_jax/models/ops.py``):

* :func:`ms_deform_attn_core_rows` -- same arguments as the reference (``ops.py:208-292``),
  channels-last ``value [B*H, sum(HW), D]``; ``sampler`` must be ``"cuda"`` and any other name is
  rejected with the reference's ``ValueError("unknown sampler ...")`` (``ops.py:235-238``);
* :func:`ms_deform_attn_core` -- the ``[B, H, D, sum(HW)]`` entry point (``ops.py:295-314``);
* :func:`ms_deform_attn` -- the signature of the drop-in contract,
  ``(value, spatial_shapes, level_start_index, sampling_locations, attention_weights)``;
* :func:`msda_prologue` -- the query -> (locations, weights) prologue of ``MSDeformAttn``
  (``ops.py:381-404``) in one launch.

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
    flat = [v for hw in shapes for v in hw]
    ws_bytes = lib.rfdetr_msda_backward_workspace_bytes(N.dtype_code(value.dtype), N.dtype_code(attention_weights.dtype),
                                                        N.int64_array(flat), batch, heads, dim, len_query, levels,
                                                        points)
    workspace = torch.empty(max(int(ws_bytes), 1), dtype=torch.uint8, device=value.device) if ws_bytes else None
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


def _prologue_launch(query, reference_points, shapes, weight, bias, n_heads, n_levels, n_points, keep_offsets):
    """One forward launch; also returns the biased offsets ``[B*Lq, 2*H*L*P]`` (float32) when
    ``keep_offsets`` (the box form's backward needs them), else None."""
    batch, len_query, channels = query.shape
    dev = query.device
    loc = torch.empty((batch, len_query, n_heads, n_levels, n_points, 2), dtype=torch.float32, device=dev)
    attn = torch.empty((batch, len_query, n_heads, n_levels * n_points), dtype=query.dtype, device=dev)
    offsets = (torch.empty((batch * len_query, 2 * n_heads * n_levels * n_points), dtype=torch.float32, device=dev)
               if keep_offsets else None)
    status = N.lib().rfdetr_msda_prologue(
        N.stream_of(query), N.ptr(query), N.dtype_code(query.dtype), N.ptr(weight), N.ptr(bias),
        N.ptr(reference_points), reference_points.shape[-1], N.int64_array([v for hw in shapes for v in hw]),
        N.ptr(loc), N.ptr(attn), N.ptr(offsets) if offsets is not None else None, batch, len_query, channels,
        n_heads, n_levels, n_points)
    N.check(status, "rfdetr_msda_prologue")
    return loc, attn, offsets


_ONES: dict = {}


def _ones(n: int, device, dtype=torch.float32) -> torch.Tensor:
    """A cached vector of n ones on `device`."""
    key = (n, str(device), dtype)
    t = _ONES.get(key)
    if t is None:
        t = _ONES[key] = torch.ones(n, device=device, dtype=dtype)
    return t


def projection_backward(g_y: torch.Tensor, query: torch.Tensor, weight: torch.Tensor):
    """The Linear layer's gradients from the projection's gradient ``g_y [B*Lq, H*L*P*3]`` (in the
    query dtype, as ``rfdetr_msda_prologue_backward`` writes it): ``(d query [B*Lq, C], d weight,
    d bias)``.  For bf16 queries these are the reference's own bf16 products -- JAX
    differentiates its bf16 ``einsum`` (``layers.py:276``) into bf16 dot products with float32
    accumulation and a bf16 cotangent -- so they run as bf16 tensor-core GEMMs (cuBLAS); the bias
    gradient is the column sum, as a matrix-vector product (a column reduction of this narrow
    matrix does not reach full bandwidth).  float32 queries keep float32 GEMMs."""
    x = query.reshape(-1, query.shape[-1])
    ones = _ones(g_y.shape[0], g_y.device, g_y.dtype)
    g_bias = torch.mv(g_y.t(), ones).float()
    g_query = torch.matmul(g_y, weight.to(g_y.dtype)).to(query.dtype)
    g_weight = torch.matmul(g_y.t(), x.to(g_y.dtype)).to(weight.dtype)
    return g_query, g_weight, g_bias


class MSDeformAttnPrologueFunction(torch.autograd.Function):
    """Forward: one ``rfdetr_msda_prologue`` launch.  Backward (with respect to the query, both
    projections and the reference points) from the saved attention weights: one
    ``rfdetr_msda_prologue_backward`` launch for the softmax and location derivatives, then the
    projection's two GEMMs (:func:`projection_backward`, cuBLAS)."""

    @staticmethod
    def forward(ctx, query, reference_points, weight, bias, shapes, n_heads, n_levels, n_points):
        # The box form's size gradient needs the forward's biased offsets: the launch keeps them.
        keep = reference_points.shape[-1] == 4 and any(ctx.needs_input_grad[:4])
        loc, attn, offsets = _prologue_launch(query, reference_points, shapes, weight, bias, n_heads, n_levels,
                                              n_points, keep)
        ctx.save_for_backward(query, reference_points, weight, attn, offsets)
        ctx.geom = (shapes, n_heads, n_levels, n_points)
        return loc, attn

    @staticmethod
    def backward(ctx, g_loc, g_attn):
        query, ref, weight, attn, offsets = ctx.saved_tensors
        shapes, H, L, P = ctx.geom
        B, Lq, C = query.shape
        hlp = H * L * P
        dev = query.device
        g_loc = (torch.zeros((B, Lq, H, L, P, 2), dtype=torch.float32, device=dev) if g_loc is None
                 else g_loc.to(torch.float32).contiguous())
        g_attn = torch.zeros_like(attn) if g_attn is None else g_attn.to(attn.dtype).contiguous()
        g_y = torch.empty((B * Lq, 3 * hlp), dtype=query.dtype, device=dev)
        g_ref = torch.empty_like(ref)
        status = N.lib().rfdetr_msda_prologue_backward(
            N.stream_of(g_loc), N.ptr(g_loc), N.ptr(g_attn), N.ptr(attn), N.dtype_code(attn.dtype), N.ptr(ref),
            ref.shape[-1], N.ptr(offsets) if offsets is not None else None,
            N.int64_array([v for hw in shapes for v in hw]), N.ptr(g_y), N.dtype_code(g_y.dtype), N.ptr(g_ref), B,
            Lq, H, L, P)
        N.check(status, "rfdetr_msda_prologue_backward")
        g_query, g_weight, g_bias = projection_backward(g_y, query, weight)
        return g_query.reshape(B, Lq, C), g_ref, g_weight, g_bias, None, None, None, None


def msda_prologue(query: torch.Tensor, reference_points: torch.Tensor, spatial_shapes, sampling_offsets_weight,
                  sampling_offsets_bias, attention_weights_weight, attention_weights_bias, n_heads: int,
                  n_levels: int, n_points: int):
    """The prologue of ``MSDeformAttn.__call__`` (``ops.py:381-404``) in one launch: the
    ``sampling_offsets`` and ``attention_weights`` Linear layers on ``query [B, Lq, C]``, the
    softmax over ``L*P`` and the location arithmetic for point (``[B, Lq, L, 2]``) or box
    (``[B, Lq, L, 4]``) reference points.  Weights use torch's Linear layout ``[out, in]`` (the
    reference's too, ``layers.py:258-280``) and are cast to the query dtype as the reference does.

    Returns ``(sampling_locations [B, Lq, H, L, P, 2] float32, attention_weights [B, Lq, H, L*P]
    in the query dtype)`` -- the sampler's inputs.
    """
    N.require_cuda(query, reference_points, sampling_offsets_weight, attention_weights_weight)
    shapes = _shapes_tuple(spatial_shapes)
    if query.dim() != 3 or len(shapes) != n_levels or reference_points.shape[:3] != (*query.shape[:2], n_levels) \
            or reference_points.shape[-1] not in (2, 4):
        raise ValueError("inconsistent shapes for msda_prologue")
    if query.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("query must be float32 or bfloat16")
    hlp = n_heads * n_levels * n_points
    weight = torch.cat([sampling_offsets_weight, attention_weights_weight], 0).to(query.dtype).contiguous()
    bias = torch.cat([sampling_offsets_bias, attention_weights_bias], 0).to(torch.float32).contiguous()
    if weight.shape != (3 * hlp, query.shape[-1]):
        raise ValueError("projection weights must be [H*L*P*2, C] and [H*L*P, C]")
    return MSDeformAttnPrologueFunction.apply(query.contiguous(), reference_points.to(torch.float32).contiguous(),
                                              weight, bias, shapes, n_heads, n_levels, n_points)

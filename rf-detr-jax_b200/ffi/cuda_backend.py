"""JAX side of the B200 backend: registers the XLA FFI handlers of ``rfdetr_ffi.cc`` and wraps
them as drop-ins for the reference's hot-path calls.  A maintainer adds this module to the
reference as ``src/rfdetr_jax/models/cuda_backend.py``.

NOT IMPORTED OR RUN IN THIS REPOSITORY: JAX is absent from this image and from the GPU hosts (the
package's own host layer binds the same C entry points through ctypes and PyTorch instead).  The
tests only check that this file parses and that every handler it names is defined in
``rfdetr_ffi.cc``.

Call sites (reference file:line) and the switch each takes:

* ``ops.py:235-238`` -- ``sampler == "cuda"``: ``return sample_cuda(value, spatial_shapes,
  sampling_locations, attention_weights)`` before the level loop;
* ``ops.py:381-404`` -- ``sampler == "cuda"``: ``loc, attn = msda_prologue(query, reference_points,
  spatial_shapes, w, b, n_heads, n_points)`` in place of the two Linear layers, the location
  arithmetic and the softmax;
* ``transformer.py:696`` -- ``_, topk_indices = top_k(proposal_scores, topk)``;
* ``postprocess.py:40`` -- ``scores, indexes = top_k(probabilities, k)``;
* ``criterion.py:79-90`` -- ``matcher == "cuda"``: ``return hungarian_match(cost, sizes, group_detr)``
  (no host callback: it runs per shard inside ``shard_map``, lifting ``run.py:479-480``);
* ``criterion.py:402-413`` -- ``matcher == "cuda"``: one ``match_stacked`` call for the stacked
  layer costs and the solve.
"""

from __future__ import annotations

import ctypes
import functools
import os

import jax
import jax.numpy as jnp
import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_lib = ctypes.cdll.LoadLibrary(os.environ.get("RFDETR_FFI_LIB", os.path.join(_HERE, "librfdetr_ffi.so")))

HANDLERS = ("RfdetrMsdaFwd", "RfdetrMsdaBwd", "RfdetrMsdaBwdNoAlloc", "RfdetrMsdaPrologue", "RfdetrMsdaPrologueBwd",
            "RfdetrTopkSelect", "RfdetrSelectRows", "RfdetrMatchCost", "RfdetrLsapBatched", "RfdetrMatchStacked",
            "RfdetrSetLosses")
for _name in HANDLERS:
    jax.ffi.register_ffi_target(_name, jax.ffi.pycapsule(getattr(_lib, _name)), platform="CUDA")


def _flat_shapes(spatial_shapes):
    return np.asarray([v for hw in spatial_shapes for v in hw], np.int64)


# ---- sampler ---------------------------------------------------------------------------------
@functools.partial(jax.custom_vjp, nondiff_argnums=(1,))  # the pattern of deform_pallas.py:132-178
def sample_cuda(value, spatial_shapes, sampling_locations, attention_weights):
    """``ms_deform_attn_core_rows(value, spatial_shapes, loc, w, "cuda")`` (``ops.py:208-292``)."""
    b, lq, h = sampling_locations.shape[:3]
    out = jax.ShapeDtypeStruct((b, lq, h * value.shape[-1]), jnp.result_type(value.dtype, attention_weights.dtype))
    return jax.ffi.ffi_call("RfdetrMsdaFwd", out)(value, sampling_locations.astype(jnp.float32), attention_weights,
                                                  spatial_shapes=_flat_shapes(spatial_shapes))


def _sample_fwd(value, spatial_shapes, loc, weights):
    return sample_cuda(value, spatial_shapes, loc, weights), (value, loc, weights)


def _sample_bwd(spatial_shapes, residuals, g):
    value, loc, weights = residuals
    shapes = (jax.ShapeDtypeStruct(value.shape, value.dtype), jax.ShapeDtypeStruct(loc.shape, jnp.float32),
              jax.ShapeDtypeStruct(weights.shape, weights.dtype))
    gv, gl, gw = jax.ffi.ffi_call("RfdetrMsdaBwd", shapes)(value, loc.astype(jnp.float32), weights, g,
                                                           spatial_shapes=_flat_shapes(spatial_shapes))
    return gv, gl.astype(loc.dtype), gw  # cast back as deform_pallas.py:175 does


sample_cuda.defvjp(_sample_fwd, _sample_bwd)


# ---- prologue --------------------------------------------------------------------------------
@functools.partial(jax.custom_vjp, nondiff_argnums=(2, 5, 6))
def msda_prologue(query, reference_points, spatial_shapes, weight, bias, n_heads, n_points):
    """``ops.py:381-404``: ``weight`` is ``concat([sampling_offsets.weight, attention_weights.weight])``
    ``[H*L*P*3, C]`` and ``bias`` the concatenated biases."""
    return _prologue_call(query, reference_points, spatial_shapes, weight, bias, n_heads, n_points)[:2]


def _prologue_call(query, reference_points, spatial_shapes, weight, bias, n_heads, n_points):
    b, lq = query.shape[:2]
    n_levels = len(spatial_shapes)
    hlp = n_heads * n_levels * n_points
    outs = (jax.ShapeDtypeStruct((b, lq, n_heads, n_levels, n_points, 2), jnp.float32),
            jax.ShapeDtypeStruct((b, lq, n_heads, n_levels * n_points), query.dtype),
            jax.ShapeDtypeStruct((b * lq, 2 * hlp), jnp.float32))
    return jax.ffi.ffi_call("RfdetrMsdaPrologue", outs)(
        query, weight.astype(query.dtype), bias.astype(jnp.float32), reference_points.astype(jnp.float32),
        spatial_shapes=_flat_shapes(spatial_shapes), n_heads=np.int64(n_heads), n_points=np.int64(n_points))


def _prologue_fwd(query, reference_points, spatial_shapes, weight, bias, n_heads, n_points):
    loc, attn, offsets = _prologue_call(query, reference_points, spatial_shapes, weight, bias, n_heads, n_points)
    return (loc, attn), (query, reference_points, weight, bias, attn, offsets)


def _prologue_bwd(spatial_shapes, n_heads, n_points, residuals, cotangents):
    query, ref, weight, bias, attn, offsets = residuals
    g_loc, g_attn = cotangents
    b, lq, c = query.shape
    hlp = n_heads * len(spatial_shapes) * n_points
    if ref.shape[-1] != 4:
        offsets = jnp.zeros((0,), jnp.float32)
    # The projection's cotangent in the query dtype, as JAX's autodiff of the bf16 Linear has it.
    outs = (jax.ShapeDtypeStruct((b * lq, 3 * hlp), query.dtype), jax.ShapeDtypeStruct(ref.shape, jnp.float32))
    g_y, g_ref = jax.ffi.ffi_call("RfdetrMsdaPrologueBwd", outs)(
        g_loc.astype(jnp.float32), g_attn.astype(attn.dtype), attn, ref.astype(jnp.float32), offsets,
        spatial_shapes=_flat_shapes(spatial_shapes))
    x = query.reshape(b * lq, c)
    w = weight.astype(query.dtype)
    g_query = jnp.matmul(g_y, w, preferred_element_type=jnp.float32).reshape(b, lq, c).astype(query.dtype)
    g_weight = jnp.matmul(g_y.T, x, preferred_element_type=jnp.float32).astype(weight.dtype)
    g_bias = g_y.astype(jnp.float32).sum(0).astype(bias.dtype)
    return g_query, g_ref.astype(ref.dtype), g_weight, g_bias


msda_prologue.defvjp(_prologue_fwd, _prologue_bwd)


# ---- selection -------------------------------------------------------------------------------
def top_k(scores, k):
    """``jax.lax.top_k(scores, k)`` over the last axis: descending, lower index first on ties."""
    lead, n = scores.shape[:-1], scores.shape[-1]
    rows = int(np.prod(lead)) if lead else 1
    outs = (jax.ShapeDtypeStruct((rows, n), jnp.float32), jax.ShapeDtypeStruct((rows, k), jnp.float32),
            jax.ShapeDtypeStruct((rows, k), jnp.int32))
    _, values, indices = jax.ffi.ffi_call("RfdetrTopkSelect", outs)(
        scores.astype(jnp.float32).reshape(rows, n, 1), k=np.int64(k))
    return values.reshape(*lead, k).astype(scores.dtype), indices.reshape(*lead, k)


def two_stage_topk(logits, k):
    """``logits.max(-1)`` and ``jax.lax.top_k`` fused (``transformer.py:695-696``)."""
    lead, n, c = logits.shape[:-2], logits.shape[-2], logits.shape[-1]
    rows = int(np.prod(lead)) if lead else 1
    outs = (jax.ShapeDtypeStruct((rows, n), jnp.float32), jax.ShapeDtypeStruct((rows, k), jnp.float32),
            jax.ShapeDtypeStruct((rows, k), jnp.int32))
    scores, values, indices = jax.ffi.ffi_call("RfdetrTopkSelect", outs)(
        logits.astype(jnp.float32).reshape(rows, n, c), k=np.int64(k))
    return scores.reshape(*lead, n), values.reshape(*lead, k), indices.reshape(*lead, k)


def select_rows(values, indices):
    """``select_rows`` (``layers.py:225-244``) for ``values [..., N, W]`` and ``indices [..., K]``."""
    lead, n, w = values.shape[:-2], values.shape[-2], values.shape[-1]
    rows, k = int(np.prod(lead)) if lead else 1, indices.shape[-1]
    outs = (jax.ShapeDtypeStruct((rows, k, w), values.dtype), jax.ShapeDtypeStruct((1,), jnp.int32))
    out, _ = jax.ffi.ffi_call("RfdetrSelectRows", outs)(values.reshape(rows, n, w),
                                                        indices.astype(jnp.int32).reshape(rows, k))
    return out.reshape(*lead, k, w)


# ---- matcher ---------------------------------------------------------------------------------
def _cost_attrs(cost_class, cost_bbox, cost_giou, focal_alpha):
    return dict(cost_class=np.float32(cost_class), cost_bbox=np.float32(cost_bbox), cost_giou=np.float32(cost_giou),
                focal_alpha=np.float32(focal_alpha))


def build_cost_matrix(pred_logits, pred_boxes, target_labels, target_boxes, target_mask, cost_class, cost_bbox,
                      cost_giou, focal_alpha):
    """``build_cost_matrix`` for the class and box terms (``matcher.py:44-141``)."""
    b, q, _ = pred_logits.shape
    out = jax.ShapeDtypeStruct((b, q, target_labels.shape[1]), jnp.float32)
    return jax.ffi.ffi_call("RfdetrMatchCost", out)(
        pred_logits, pred_boxes, target_labels.astype(jnp.int32), target_boxes.astype(jnp.float32),
        target_mask.astype(jnp.uint8), **_cost_attrs(cost_class, cost_bbox, cost_giou, focal_alpha))


def hungarian_match(cost, sizes, group_detr):
    """``hungarian_match`` (``matcher.py:182-208``) on the device: ``(rows, cols, valid)``, each
    ``[..., B, group_detr * T]``.  The status word (a solve that hit its iteration cap, never for
    finite costs) is dropped here; a debug build can return it and check it outside the step."""
    lead = cost.shape[:-3]
    b, q, t = cost.shape[-3:]
    folded = jax.lax.stop_gradient(cost).astype(jnp.float32).reshape(-1, q, t)
    folded_sizes = jnp.broadcast_to(sizes.astype(jnp.int32), (*lead, b)).reshape(-1)
    n, slots = folded.shape[0], group_detr * t
    outs = (jax.ShapeDtypeStruct((n, slots), jnp.int32), jax.ShapeDtypeStruct((n, slots), jnp.int32),
            jax.ShapeDtypeStruct((n, slots), jnp.uint8), jax.ShapeDtypeStruct((1,), jnp.int32))
    rows, cols, valid, _ = jax.ffi.ffi_call("RfdetrLsapBatched", outs)(folded, folded_sizes,
                                                                      group_detr=np.int64(group_detr))
    shape = (*lead, b, slots)
    return rows.reshape(shape), cols.reshape(shape), valid.astype(bool).reshape(shape)


def match_stacked(pred_logits, pred_boxes, target_labels, target_boxes, target_mask, sizes, group_detr, cost_class,
                  cost_bbox, cost_giou, focal_alpha):
    """The stacked ``layer_cost`` + one solve of ``compute_losses`` (``criterion.py:402-413``):
    ``pred_logits [L, B, Q, C]`` -> ``(cost, rows, cols, valid)``."""
    lyr, b, q, _ = pred_logits.shape
    t = target_labels.shape[1]
    slots = group_detr * t
    outs = (jax.ShapeDtypeStruct((lyr, b, q, t), jnp.float32), jax.ShapeDtypeStruct((lyr, b, slots), jnp.int32),
            jax.ShapeDtypeStruct((lyr, b, slots), jnp.int32), jax.ShapeDtypeStruct((lyr, b, slots), jnp.uint8),
            jax.ShapeDtypeStruct((1,), jnp.int32))
    cost, rows, cols, valid, _ = jax.ffi.ffi_call("RfdetrMatchStacked", outs)(
        jax.lax.stop_gradient(pred_logits), jax.lax.stop_gradient(pred_boxes), target_labels.astype(jnp.int32),
        target_boxes.astype(jnp.float32), target_mask.astype(jnp.uint8), sizes.astype(jnp.int32),
        group_detr=np.int64(group_detr), **_cost_attrs(cost_class, cost_bbox, cost_giou, focal_alpha))
    return cost, rows, cols, valid.astype(bool)


# ---- set losses ------------------------------------------------------------------------------
@functools.partial(jax.custom_vjp, nondiff_argnums=(7, 8))
def set_losses(pred_logits, pred_boxes, target_labels, target_boxes, rows, cols, valid, focal_alpha, ia_bce,
               num_boxes=None):
    """``loss_labels`` + ``loss_boxes`` of stacked layers (``criterion.py:157-250``): ``[L, 3]``
    losses (classification, L1, GIoU)."""
    return _set_losses_call(pred_logits, pred_boxes, target_labels, target_boxes, rows, cols, valid, focal_alpha,
                            ia_bce, num_boxes)[0]


def _set_losses_call(pred_logits, pred_boxes, target_labels, target_boxes, rows, cols, valid, focal_alpha, ia_bce,
                     num_boxes):
    lyr, b, q, c = pred_logits.shape
    outs = (jax.ShapeDtypeStruct((lyr, 3), jnp.float32), jax.ShapeDtypeStruct((lyr, b, q, c), jnp.float32),
            jax.ShapeDtypeStruct((lyr, b, q, 4), jnp.float32), jax.ShapeDtypeStruct((lyr, b, q, 4), jnp.float32))
    nb = jnp.ones((1,), jnp.float32) if num_boxes is None else jnp.reshape(num_boxes, (1,)).astype(jnp.float32)
    return jax.ffi.ffi_call("RfdetrSetLosses", outs)(
        pred_logits.astype(jnp.float32), pred_boxes.astype(jnp.float32), target_labels.astype(jnp.int32),
        target_boxes.astype(jnp.float32), rows.astype(jnp.int32), cols.astype(jnp.int32), valid.astype(jnp.uint8), nb,
        focal_alpha=np.float32(focal_alpha), ia_bce=np.int32(1 if ia_bce else 0))


def _set_losses_fwd(pred_logits, pred_boxes, target_labels, target_boxes, rows, cols, valid, focal_alpha, ia_bce,
                    num_boxes=None):
    losses, g_logits, g_l1, g_giou = _set_losses_call(pred_logits, pred_boxes, target_labels, target_boxes, rows,
                                                      cols, valid, focal_alpha, ia_bce, num_boxes)
    return losses, (g_logits, g_l1, g_giou, pred_logits.dtype, pred_boxes.dtype)


def _set_losses_bwd(focal_alpha, ia_bce, residuals, g):
    g_logits, g_l1, g_giou, logits_dtype, boxes_dtype = residuals
    scale = g[:, 0].reshape(-1, 1, 1, 1)
    d_logits = (g_logits * scale).astype(logits_dtype)
    d_boxes = (g_l1 * g[:, 1].reshape(-1, 1, 1, 1) + g_giou * g[:, 2].reshape(-1, 1, 1, 1)).astype(boxes_dtype)
    return d_logits, d_boxes, None, None, None, None, None, None


set_losses.defvjp(_set_losses_fwd, _set_losses_bwd)

"""CPU oracle for the multi-scale deformable-attention sampler -- TEST INFRASTRUCTURE.

Restates the reference's ``"gather"`` sampler (``src/rfdetr_jax/models/ops.py``) in NumPy:

* sample coordinates: ``grids = 2 * loc - 1`` in at least float32 (``ops.py:270``), then
  ``ix = ((gx + 1) * W - 1) / 2`` (``ops.py:83-84``), every step an IEEE float32 operation in
  the reference's order, so ``floor(ix)`` -- the one discontinuous step -- agrees bit for bit;
* bilinear taps: ``floor``, fractional weights, the four corners in the order
  ``(x0,y0), (x1,y0), (x0,y1), (x1,y1)``, in-bounds masks and clipped indices
  (``ops.py:85-106,110-128``); out-of-bounds taps contribute zero (``padding_mode="zeros"``);
* the level loop and the weighted sum over ``L * P`` points (``ops.py:265-292``);
* the backward pass is the analytic gradient of that gather path, which is what JAX autodiff
  of it computes: ``floor`` has zero derivative, masked taps contribute nothing, and
  ``d ix / d loc = W`` (``ops.py:83`` with ``ops.py:270``).  The same formulas appear in the
  reference's fused kernel (``deform_pallas.py:97-120``: ``da = sum_d g*s``,
  ``dix = a * sum_d g * (V dK/dx)``, ``dV += (g*a) K^T``).

Accumulation runs in float64 (``compute=np.float64``, the parity oracle) or float32
(``compute=np.float32``, the timed CPU baseline).  The bf16 path of the reference rounds its
interpolation weights to bf16 (``ops.py:88-89``); the oracle keeps them exact, as the
reference's fused kernel does (``deform_pallas.py:91``), and the bf16 tolerance covers the gap.

Non-finite sampling locations give NaN outputs and gradients (the reference's
``ix - floor(ix)`` is NaN there); they add nothing to ``grad_value``.

Work is done one image at a time so the full-size training shape (config 2) fits in memory.
"""

from __future__ import annotations

import numpy as np

_ONE = np.float32(1.0)
_TWO = np.float32(2.0)


def coordinates(loc_x: np.ndarray, loc_y: np.ndarray, height: int, width: int):
    """Pixel coordinates ``(ix, iy)`` in float32, in the reference's exact op order.

    ``ops.py:270``: ``grids = 2 * loc - 1``; ``ops.py:83-84``: ``ix = ((gx + 1) * W - 1) / 2``.
    """
    loc_x = np.asarray(loc_x, np.float32)
    loc_y = np.asarray(loc_y, np.float32)
    gx = _TWO * loc_x - _ONE
    gy = _TWO * loc_y - _ONE
    ix = ((gx + _ONE) * np.float32(width) - _ONE) / _TWO
    iy = ((gy + _ONE) * np.float32(height) - _ONE) / _TWO
    return ix, iy


def bilinear_taps(ix: np.ndarray, iy: np.ndarray, height: int, width: int, compute=np.float64):
    """The four bilinear taps of every sample (``ops.py:85-128``).

    Returns:
        ``(index, weight, d_weight_dx, d_weight_dy)``, each ``[4, *ix.shape]``: the clipped
        flat corner index ``y * W + x``, the masked tap weight, and the masked weight's
        derivatives with respect to ``ix`` and ``iy``.  Corner order is
        ``(x0,y0), (x1,y0), (x0,y1), (x1,y1)`` as at ``ops.py:110-117``.
    """
    finite = np.isfinite(ix) & np.isfinite(iy)
    safe_ix = np.where(finite, ix, np.float32(-4.0))
    safe_iy = np.where(finite, iy, np.float32(-4.0))
    ix0 = np.floor(safe_ix)
    iy0 = np.floor(safe_iy)
    # ix - floor(ix) is exact in float32; widen afterwards.
    wx1 = (safe_ix - ix0).astype(compute)
    wy1 = (safe_iy - iy0).astype(compute)
    wx0 = compute(1.0) - wx1
    wy0 = compute(1.0) - wy1

    # Clamp before the integer conversion so far-off positions cannot overflow int64.
    ix0i = np.clip(ix0, -2.0, width + 1.0).astype(np.int64)
    iy0i = np.clip(iy0, -2.0, height + 1.0).astype(np.int64)
    ix1i = ix0i + 1
    iy1i = iy0i + 1
    in_x0 = (ix0i >= 0) & (ix0i < width)
    in_x1 = (ix1i >= 0) & (ix1i < width)
    in_y0 = (iy0i >= 0) & (iy0i < height)
    in_y1 = (iy1i >= 0) & (iy1i < height)
    x0c = np.clip(ix0i, 0, width - 1)
    x1c = np.clip(ix1i, 0, width - 1)
    y0c = np.clip(iy0i, 0, height - 1)
    y1c = np.clip(iy1i, 0, height - 1)

    index = np.stack([y0c * width + x0c, y0c * width + x1c, y1c * width + x0c, y1c * width + x1c])
    inside = np.stack([in_x0 & in_y0, in_x1 & in_y0, in_x0 & in_y1, in_x1 & in_y1]).astype(compute)
    weight = np.stack([wx0 * wy0, wx1 * wy0, wx0 * wy1, wx1 * wy1]) * inside
    d_dx = np.stack([-wy0, wy0, -wy1, wy1]) * inside
    d_dy = np.stack([-wx0, -wx1, wx0, wx1]) * inside
    nan = ~finite
    if nan.any():
        weight[:, nan] = np.nan
        d_dx[:, nan] = np.nan
        d_dy[:, nan] = np.nan
    return index, weight, d_dx, d_dy


def _check(value, spatial_shapes, loc, attn):
    value = np.asarray(value)
    loc = np.asarray(loc)
    attn = np.asarray(attn)
    if loc.ndim != 6 or loc.shape[-1] != 2:
        raise ValueError("sampling_locations must be [B, Lq, H, L, P, 2]")
    batch, len_query, heads, levels, points, _ = loc.shape
    if len(spatial_shapes) != levels:
        raise ValueError("spatial_shapes must have one (H, W) pair per level")
    total = sum(int(h) * int(w) for h, w in spatial_shapes)
    if value.ndim != 3 or value.shape[0] != batch * heads or value.shape[1] != total:
        raise ValueError("value must be [B * H, sum(H*W), D]")
    if attn.shape != (batch, len_query, heads, levels * points):
        raise ValueError("attention_weights must be [B, Lq, H, L * P]")
    return batch, len_query, heads, levels, points, value.shape[2]


def _level_offsets(spatial_shapes):
    offsets = [0]
    for height, width in spatial_shapes:
        offsets.append(offsets[-1] + int(height) * int(width))
    return offsets


def forward_image(value_b, spatial_shapes, loc_b, attn_b, compute=np.float64):
    """One image of ``ms_deform_attn_core_rows`` (``ops.py:265-292``).

    Args:
        value_b: ``[H, sum(HW), D]`` (the image's rows of the ``[B*H, ...]`` value tensor).
        loc_b: ``[Lq, H, L, P, 2]`` float32.
        attn_b: ``[Lq, H, L*P]``.

    Returns:
        ``[Lq, H*D]`` in ``compute`` precision.
    """
    heads, _, dim = value_b.shape
    len_query, _, levels, points, _ = loc_b.shape
    value_b = np.asarray(value_b, compute)
    weights = np.asarray(attn_b, compute).reshape(len_query, heads, levels, points).transpose(1, 0, 2, 3)
    offsets = _level_offsets(spatial_shapes)
    out = np.zeros((heads, len_query, dim), compute)
    for level, (height, width) in enumerate(spatial_shapes):
        level_value = value_b[:, offsets[level]:offsets[level + 1], :]
        xy = np.asarray(loc_b[:, :, level], np.float32).transpose(1, 0, 2, 3)  # [H, Lq, P, 2]
        ix, iy = coordinates(xy[..., 0], xy[..., 1], height, width)
        index, weight, _, _ = bilinear_taps(ix, iy, height, width, compute)
        sampled = np.zeros(ix.shape + (dim,), compute)
        for corner in range(4):
            flat = index[corner].reshape(heads, -1)
            taken = level_value[np.arange(heads)[:, None], flat].reshape(ix.shape + (dim,))
            sampled += weight[corner][..., None] * taken
        out += np.einsum("hqp,hqpd->hqd", weights[:, :, level], sampled)
    return out.transpose(1, 0, 2).reshape(len_query, heads * dim)


def backward_image(value_b, spatial_shapes, loc_b, attn_b, grad_b, compute=np.float64):
    """Gradients of one image's sampler output with respect to value, locations and weights.

    Args:
        grad_b: ``[Lq, H*D]`` cotangent of the output.

    Returns:
        ``(grad_value [H, sum(HW), D], grad_loc [Lq, H, L, P, 2], grad_attn [Lq, H, L*P])``.
    """
    heads, total, dim = value_b.shape
    len_query, _, levels, points, _ = loc_b.shape
    value_b = np.asarray(value_b, compute)
    weights = np.asarray(attn_b, compute).reshape(len_query, heads, levels, points).transpose(1, 0, 2, 3)
    grad = np.asarray(grad_b, compute).reshape(len_query, heads, dim).transpose(1, 0, 2)  # [H, Lq, D]
    offsets = _level_offsets(spatial_shapes)
    grad_value = np.zeros((heads * total, dim), compute)
    grad_loc = np.zeros((heads, len_query, levels, points, 2), compute)
    grad_attn = np.zeros((heads, len_query, levels, points), compute)
    rows = np.arange(heads)[:, None]
    for level, (height, width) in enumerate(spatial_shapes):
        level_value = value_b[:, offsets[level]:offsets[level + 1], :]
        xy = np.asarray(loc_b[:, :, level], np.float32).transpose(1, 0, 2, 3)  # [H, Lq, P, 2]
        ix, iy = coordinates(xy[..., 0], xy[..., 1], height, width)
        index, weight, d_dx, d_dy = bilinear_taps(ix, iy, height, width, compute)
        shape = ix.shape + (dim,)
        taken = [level_value[rows, index[c].reshape(heads, -1)].reshape(shape) for c in range(4)]
        sampled = sum(weight[c][..., None] * taken[c] for c in range(4))
        along_x = sum(d_dx[c][..., None] * taken[c] for c in range(4))
        along_y = sum(d_dy[c][..., None] * taken[c] for c in range(4))
        a = weights[:, :, level]  # [H, Lq, P]
        g = grad[:, :, None, :]  # [H, Lq, 1, D]
        grad_attn[:, :, level] = (g * sampled).sum(-1)
        grad_loc[:, :, level, :, 0] = a * (g * along_x).sum(-1) * compute(width)
        grad_loc[:, :, level, :, 1] = a * (g * along_y).sum(-1) * compute(height)
        scaled = a[..., None] * g  # [H, Lq, P, D]
        base = (np.arange(heads) * total + offsets[level])[:, None, None]
        for c in range(4):
            contribution = np.where(np.isfinite(weight[c])[..., None], weight[c][..., None] * scaled, 0.0)
            flat = (base + index[c]).ravel()
            for d in range(dim):
                grad_value[:, d] += np.bincount(flat, weights=contribution[..., d].ravel(),
                                                minlength=heads * total)
    return (
        grad_value.reshape(heads, total, dim),
        grad_loc.transpose(1, 0, 2, 3, 4),
        grad_attn.transpose(1, 0, 2, 3).reshape(len_query, heads, levels * points),
    )


def ms_deform_attn_forward(value, spatial_shapes, loc, attn, compute=np.float64):
    """``ms_deform_attn_core_rows(value, spatial_shapes, loc, attn)`` (``ops.py:208-292``).

    Args:
        value: ``[B*H, sum(HW), D]``; loc: ``[B, Lq, H, L, P, 2]``; attn: ``[B, Lq, H, L*P]``.

    Returns:
        ``[B, Lq, H*D]`` in ``compute`` precision.
    """
    batch, len_query, heads, _, _, dim = _check(value, spatial_shapes, loc, attn)
    value = np.asarray(value)
    out = np.empty((batch, len_query, heads * dim), compute)
    for b in range(batch):
        out[b] = forward_image(value[b * heads:(b + 1) * heads], spatial_shapes, loc[b], attn[b], compute)
    return out


def ms_deform_attn_backward(value, spatial_shapes, loc, attn, grad_out, compute=np.float64):
    """Gradients ``(grad_value, grad_loc, grad_attn)`` of the sampler output against ``grad_out``."""
    batch, len_query, heads, levels, points, dim = _check(value, spatial_shapes, loc, attn)
    value = np.asarray(value)
    grad_value = np.empty(value.shape, compute)
    grad_loc = np.empty(np.shape(loc), compute)
    grad_attn = np.empty(np.shape(attn), compute)
    for b in range(batch):
        gv, gl, ga = backward_image(value[b * heads:(b + 1) * heads], spatial_shapes, loc[b], attn[b],
                                    grad_out[b], compute)
        grad_value[b * heads:(b + 1) * heads] = gv
        grad_loc[b] = gl
        grad_attn[b] = ga
    return grad_value, grad_loc, grad_attn


def forward_bf16_gather(value, spatial_shapes, loc, attn):
    """The reference's ``"gather"`` sampler on bf16 activations with the roundings of its bf16
    graph (``ops.py:76-135`` per level, ``ops.py:264-292`` across levels), for measuring how far
    the reference's own bf16 output sits from the exact one (the timed kernels follow the fused
    kernel, ``deform_pallas.py:91``, and keep these steps in float32):

    * ``wx1 = bf16(ix - floor(ix))``, ``wy1`` likewise (``ops.py:88-89``); ``wx0 = bf16(1 - wx1)``,
      ``wy0`` likewise (``ops.py:90-91``);
    * the corner weights ``bf16(wxa * wyb)`` times the 0/1 in-bounds mask (``ops.py:121-127``);
    * each tap ``bf16(value * weight)`` and the sum of the four (``ops.py:134``);
    * the points weighted by the bf16 attention weights in one contraction (``ops.py:289``),
      rounded to bf16 once.

    The two sums are taken in a float32 accumulator and rounded once -- an assumption about how
    XLA reduces bf16 operands, which this image cannot check (JAX is absent).  ``value`` and
    ``attn`` must hold bf16 values; locations must be finite.  Returns float32 holding bf16
    values, ``[B, Lq, H*D]``.
    """
    batch, len_query, heads, levels, points, dim = _check(value, spatial_shapes, loc, attn)
    loc = np.asarray(loc, np.float32)
    if not np.isfinite(loc).all():
        raise ValueError("forward_bf16_gather takes finite locations only")
    value = np.asarray(value, np.float32)
    attn = np.asarray(attn, np.float32)
    offsets = _level_offsets(spatial_shapes)
    one = np.float32(1.0)
    out = np.empty((batch, len_query, heads * dim), np.float32)
    for b in range(batch):
        vb = value[b * heads:(b + 1) * heads]
        acc = np.zeros((heads, len_query, dim), np.float32)
        weights = attn[b].reshape(len_query, heads, levels, points).transpose(1, 0, 2, 3)  # [H, Lq, L, P]
        for level, (height, width) in enumerate(spatial_shapes):
            level_value = vb[:, offsets[level]:offsets[level + 1], :]
            xy = loc[b, :, :, level].transpose(1, 0, 2, 3)  # [H, Lq, P, 2]
            ix, iy = coordinates(xy[..., 0], xy[..., 1], height, width)
            ix0, iy0 = np.floor(ix), np.floor(iy)
            wx1, wy1 = bf16_round(ix - ix0), bf16_round(iy - iy0)
            wx0, wy0 = bf16_round(one - wx1), bf16_round(one - wy1)
            index, _, _, _ = bilinear_taps(ix, iy, height, width, np.float32)
            ix0i, iy0i = ix0.astype(np.int64), iy0.astype(np.int64)
            in_x0 = (ix0i >= 0) & (ix0i < width)
            in_x1 = (ix0i + 1 >= 0) & (ix0i + 1 < width)
            in_y0 = (iy0i >= 0) & (iy0i < height)
            in_y1 = (iy0i + 1 >= 0) & (iy0i + 1 < height)
            corner_w = [bf16_round(wx0 * wy0) * (in_x0 & in_y0), bf16_round(wx1 * wy0) * (in_x1 & in_y0),
                        bf16_round(wx0 * wy1) * (in_x0 & in_y1), bf16_round(wx1 * wy1) * (in_x1 & in_y1)]
            sampled = np.zeros(ix.shape + (dim,), np.float32)
            for corner in range(4):
                flat = index[corner].reshape(heads, -1)
                taken = level_value[np.arange(heads)[:, None], flat].reshape(ix.shape + (dim,))
                sampled += bf16_round(taken * corner_w[corner].astype(np.float32)[..., None])
            sampled = bf16_round(sampled)  # [H, Lq, P, D]
            for p in range(points):
                acc += weights[:, :, level, p][..., None] * sampled[:, :, p]
        out[b] = bf16_round(acc).transpose(1, 0, 2).reshape(len_query, heads * dim)
    return out


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), returned as float32."""
    bits = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000
    out = rounded.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), np.float32(np.nan), out)

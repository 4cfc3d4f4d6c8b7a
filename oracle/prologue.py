"""CPU oracle for the MSDA prologue (query -> sampling locations, attention weights) --
TEST INFRASTRUCTURE.

Restates the query side of ``MSDeformAttn.__call__`` (``src/rfdetr_jax/models/ops.py:381-404``)
in NumPy, with every rounding step the reference takes for a float32 or a bf16 query:

* ``Linear`` (``src/rfdetr_jax/models/layers.py:258-280``): ``y = x @ weight.astype(x.dtype).T``
  rounded to the query dtype, then ``y + bias.astype(y.dtype)`` rounded to it again.  The dot
  products are formed exactly (float64 over products of float32 or bf16 values) and rounded once;
  a float32 summation (any order) lands within ``4 sqrt(C) 2**-24 sum|x_i w_i|`` of that -- a
  random-walk bound, not the worst case -- so for a bf16 query the rounding to bf16 is
  *determined* unless a bf16 rounding midpoint lies within that distance.  :func:`prologue_forward` returns, besides the locations, the locations computed from
  the other rounding for exactly those ambiguous entries (``loc_alt``), so a test can demand one
  of the two bit for bit.
* point references (``ops.py:388-394``): ``loc = ref + precise_divide(off, (W_l, H_l))`` -- the
  bf16 offsets promoted to float32, one IEEE float32 division (``precise_divide``,
  ``ops.py:46-62``), one float32 addition;
* box references (``ops.py:395-399``): ``loc = ref_xy + precise_divide(off, P) * ref_wh * 0.5``
  -- the division by the Python int ``P`` stays in the query dtype (weak typing), computed in
  float32 and rounded to bf16 for a bf16 query; then float32 products and the sum;
* ``softmax`` of the logits promoted to float32 (``ops.py:403-404``), then cast to the query
  dtype.  The oracle evaluates it in float64 and rounds once; ``attn_tie`` marks bf16 weights
  whose float64 value lies within ``2**-20`` relative of a bf16 rounding midpoint, where a float32
  evaluation (any ``exp``) may round the other way.

:func:`prologue_backward` is the float64 gradient of the same function for given cotangents of
``(loc, attn)`` -- what JAX autodiff of ``ops.py:381-404`` computes up to float32 rounding:
``d logits = a * (g - sum(a g))``, ``d off = g_loc / (W, H)`` (points) or ``g_loc * wh * 0.5 / P``
(boxes), ``d ref_xy = sum over heads and points of g_loc``, ``d ref_wh = sum g_loc * off / P *
0.5``, then the projection's ``d query = d y @ W``, ``d W = d y^T @ query``, ``d bias = sum d y``.
Rounding casts have identity derivatives, as in JAX.

Pinning: the division and rounding steps are checked against the reference's own known answers
(``tests/test_ops.py:264-279``: ``precise_divide`` equals NumPy's float32 quotient, for an array
divisor and for the Python int 24) and against an independent torch evaluation of the same
expression; the gradient against torch float64 autograd.
"""

from __future__ import annotations

import numpy as np


def bf16_round(x) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even), returned as float32."""
    x = np.ascontiguousarray(x, np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32).copy()
    nan = np.isnan(x)
    out[nan] = x[nan]
    return out


def precise_divide(numerator, denominator) -> np.ndarray:
    """``precise_divide`` (``ops.py:46-62``) for float32 operands: one IEEE rounding."""
    return (np.asarray(numerator, np.float32) / np.asarray(denominator, np.float32)).astype(np.float32)


def _to_dtype(x, dtype: str) -> np.ndarray:
    x32 = np.asarray(x, np.float64).astype(np.float32)
    return bf16_round(x32) if dtype == "bf16" else x32


def _bf16_neighbours(exact: np.ndarray):
    """The two bf16 values around each float64 value (equal when it is a bf16 value)."""
    exact = np.asarray(exact, np.float64)
    near32 = bf16_round(exact.astype(np.float32))
    near = near32.astype(np.float64)
    bits = np.ascontiguousarray(near32).view(np.uint32).astype(np.int64)
    # Sign-magnitude bit patterns: +0x10000 moves away from zero, -0x10000 towards it.
    away = (bits + (1 << 16)).astype(np.uint32).view(np.float32).astype(np.float64)
    toward = np.maximum(bits - (1 << 16), 0).astype(np.uint32).view(np.float32).astype(np.float64)
    toward = np.where(near == 0, -np.sign(exact) * 2.0 ** -133, toward)
    other = np.where(np.abs(exact) > np.abs(near), away, toward)
    other = np.where((near == 0) & (exact != 0), np.sign(exact) * 2.0 ** -133, other)
    return near, other


def _midpoint_distance(exact: np.ndarray) -> np.ndarray:
    """Distance from each value to the nearest bf16 rounding midpoint."""
    near, other = _bf16_neighbours(exact)
    mid = 0.5 * (near + other)
    return np.abs(exact - mid)


def projection(query, weight, bias, dtype: str):
    """``Linear`` of ``layers.py:276-279`` for a float32 or bf16 query.

    Returns ``(y, y_alt, ambiguous)``: ``y`` the reference's result (projection rounded to the
    query dtype, bias rounded to it and added with one more rounding), as float32; ``y_alt`` the
    same with the projection rounded the other way where that rounding is ambiguous (``y``
    elsewhere); ``ambiguous`` marks those entries.
    """
    x = _to_dtype(query, dtype).astype(np.float64)
    w = _to_dtype(weight, dtype).astype(np.float64)
    x2 = x.reshape(-1, x.shape[-1])
    exact = x2 @ w.T
    # The rounding errors of a float32 sum add up like a random walk: 4 * sqrt(C) units of
    # sum|x_i w_i| (2**-24 each) lies far outside what any summation order produces, while the
    # worst case, (C - 1) units, would mark about 40% of the entries at C = 256.
    bound = 4.0 * np.sqrt(x2.shape[-1]) * 2.0 ** -24 * (np.abs(x2) @ np.abs(w).T)
    b = _to_dtype(bias, dtype)
    if dtype == "bf16":
        near, other = _bf16_neighbours(exact)
        ambiguous = _midpoint_distance(exact) <= bound
        y = bf16_round((near.astype(np.float32) + b).astype(np.float32))
        y_alt = bf16_round((np.where(ambiguous, other, near).astype(np.float32) + b).astype(np.float32))
    else:
        p = exact.astype(np.float32)
        y = (p + b).astype(np.float32)
        y_alt = y
        ambiguous = np.zeros(exact.shape, bool)
    shape = (*np.shape(query)[:-1], w.shape[0])
    return y.reshape(shape), y_alt.reshape(shape), ambiguous.reshape(shape)


def _locations(off, ref, shapes, n_points, dtype):
    """``ops.py:388-399`` on float32 offsets ``[B, Lq, H, L, P, 2]`` (already in the query dtype)."""
    ref = np.asarray(ref, np.float32)
    if ref.shape[-1] == 2:
        norm = np.array([[w, h] for h, w in shapes], np.float32)  # (W_l, H_l)
        q = precise_divide(off, norm[None, None, None, :, None, :])
        return (ref[:, :, None, :, None, :] + q).astype(np.float32)
    t = precise_divide(off, n_points)
    if dtype == "bf16":
        t = bf16_round(t)
    wh = ref[:, :, None, :, None, 2:]
    scaled = ((t * wh).astype(np.float32) * np.float32(0.5)).astype(np.float32)
    return (ref[:, :, None, :, None, :2] + scaled).astype(np.float32)


def prologue_forward(query, reference_points, shapes, w_off, b_off, w_att, b_att, n_heads, n_levels, n_points,
                     dtype: str = "f32"):
    """``ops.py:381-404``: returns a dict with ``loc`` (float32 ``[B, Lq, H, L, P, 2]``),
    ``loc_alt`` (the other admissible rounding, see the module docstring), ``attn`` (float32
    values of the query dtype, ``[B, Lq, H, L*P]``), ``attn_tie`` (bf16 rounding not determined
    by a float32 evaluation), ``attn_f64`` (the unrounded softmax) and the float32 ``offsets``
    (the biased projection's offsets part, ``[B, Lq, H, L, P, 2]``) with ``offsets_alt``, their other
    admissible rounding."""
    batch, len_query, _ = np.shape(query)
    hlp = n_heads * n_levels * n_points
    y, y_alt, amb = projection(query, np.concatenate([w_off, w_att], 0), np.concatenate([b_off, b_att], 0), dtype)
    off = y[..., :2 * hlp].reshape(batch, len_query, n_heads, n_levels, n_points, 2)
    off_alt = y_alt[..., :2 * hlp].reshape(off.shape)
    logits = y[..., 2 * hlp:].reshape(batch, len_query, n_heads, n_levels * n_points).astype(np.float64)
    z = np.exp(logits - logits.max(-1, keepdims=True))
    attn64 = z / z.sum(-1, keepdims=True)
    attn = _to_dtype(attn64, dtype)
    if dtype == "bf16":
        tie = _midpoint_distance(attn64) <= 2.0 ** -20 * np.abs(attn64)
    else:
        tie = np.zeros(attn.shape, bool)
    loc = _locations(off, reference_points, shapes, n_points, dtype)
    loc_alt = _locations(off_alt, reference_points, shapes, n_points, dtype)
    return {"loc": loc, "loc_alt": loc_alt, "attn": attn, "attn_tie": tie, "attn_f64": attn64, "offsets": off,
            "offsets_alt": off_alt,
            "logits_ambiguous": amb[..., 2 * hlp:].reshape(logits.shape)}


def prologue_backward(query, reference_points, shapes, w_off, b_off, w_att, b_att, n_heads, n_levels, n_points,
                      g_loc, g_attn, dtype: str = "f32"):
    """Float64 gradients ``(query, reference_points, w_off, b_off, w_att, b_att)`` of
    ``sum(loc * g_loc) + sum(attn * g_attn)``, evaluated at the reference's forward values."""
    fwd = prologue_forward(query, reference_points, shapes, w_off, b_off, w_att, b_att, n_heads, n_levels, n_points,
                           dtype)
    batch, len_query, channels = np.shape(query)
    L, P, H = n_levels, n_points, n_heads
    hlp = H * L * P
    ref = np.asarray(reference_points, np.float64)
    g_loc = np.asarray(g_loc, np.float64)
    g_attn = np.asarray(g_attn, np.float64)
    a = fwd["attn_f64"]
    d_logits = a * (g_attn - (a * g_attn).sum(-1, keepdims=True))
    off = fwd["offsets"].astype(np.float64)
    g_ref = np.zeros_like(ref)
    g_ref[..., :2] = g_loc.sum(axis=(2, 4))
    if ref.shape[-1] == 2:
        norm = np.array([[w, h] for h, w in shapes], np.float64)
        d_off = g_loc / norm[None, None, None, :, None, :]
    else:
        wh = ref[:, :, None, :, None, 2:]
        d_off = g_loc * wh * 0.5 / P
        g_ref[..., 2:] = (g_loc * off / P * 0.5).sum(axis=(2, 4))
    d_y = np.concatenate([d_off.reshape(batch * len_query, 2 * hlp), d_logits.reshape(batch * len_query, hlp)], -1)
    x = _to_dtype(query, dtype).astype(np.float64).reshape(-1, channels)
    w = _to_dtype(np.concatenate([w_off, w_att], 0), dtype).astype(np.float64)
    g_query = (d_y @ w).reshape(batch, len_query, channels)
    g_w = d_y.T @ x
    g_b = d_y.sum(0)
    return g_query, g_ref, g_w[:2 * hlp], g_b[:2 * hlp], g_w[2 * hlp:], g_b[2 * hlp:]

"""Test helpers: golden fixtures, tolerances and input generators shared by the test modules."""

from __future__ import annotations

import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# Tolerances of the parity contract.
FP32_RTOL = 1e-5  # fp32 sampler outputs and gradients: 1e-5 relative ...
FP32_ATOL = 1e-6  # ... and 1e-6 absolute, elementwise
BF16_REL = 2e-2   # bf16: 2e-2 relative (max error against the tensor's scale, and relative L2)


def unpack_bf16(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def load_golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        data = {k: z[k] for k in z.files}
    if "bf16" in data and bool(data["bf16"]):
        for key in ("value", "attn", "grad"):
            data[key] = unpack_bf16(data[key])
    if "shapes" in data:
        data["shapes"] = tuple((int(h), int(w)) for h, w in data["shapes"])
    return data


def assert_fp32_close(got, want, what="", rtol=FP32_RTOL, atol=FP32_ATOL):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} vs {want.shape}"
    err = np.abs(got - want)
    bound = atol + rtol * np.abs(want)
    bad = ~(err <= bound)
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {bad.size} elements outside |err| <= {atol} + {rtol}|ref|; "
                           f"worst err {err[bad].max():.3e} at ref {want[bad][np.argmax(err[bad])]:.3e}")


def assert_bf16_close(got, want, what="", rel=BF16_REL):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} vs {want.shape}"
    assert np.isfinite(got).all(), f"{what}: non-finite values"
    err = np.abs(got - want)
    scale = max(1.0, float(np.abs(want).max(initial=0.0)))
    assert err.max(initial=0.0) <= rel * scale, f"{what}: max err {err.max():.3e} > {rel} * {scale:.3e}"
    norm = float(np.linalg.norm(want))
    if norm > 0:
        assert np.linalg.norm(got - want) / norm <= rel, f"{what}: relative L2 {np.linalg.norm(got - want) / norm:.3e}"


def softmax(x, axis=-1):
    x = x - x.max(axis=axis, keepdims=True)
    e = np.exp(x)
    return e / e.sum(axis=axis, keepdims=True)


def sampler_inputs(seed, batch, len_query, heads, shapes, points, dim, lo=0.0, hi=1.0, sigma=1.0):
    """Seeded sampler inputs with the benchmark configs' distributions (float32 arrays)."""
    rng = np.random.default_rng(seed)
    total = sum(h * w for h, w in shapes)
    value = rng.standard_normal((batch * heads, total, dim)).astype(np.float32)
    loc = rng.uniform(lo, hi, (batch, len_query, heads, len(shapes), points, 2)).astype(np.float32)
    attn = softmax(rng.normal(0.0, sigma, (batch, len_query, heads, len(shapes) * points))).astype(np.float32)
    grad = rng.standard_normal((batch, len_query, heads * dim)).astype(np.float32)
    return value, loc, attn, grad


def match_inputs(seed, batch, queries, classes, max_targets, sizes=None):
    """Config-4 style predictions and padded targets."""
    rng = np.random.default_rng(seed)
    if sizes is None:
        sizes = rng.integers(1, max_targets + 1, batch)
    sizes = np.asarray(sizes, np.int32)
    labels = rng.integers(0, classes, (batch, max_targets)).astype(np.int32)
    tboxes = np.concatenate([rng.uniform(0.05, 0.95, (batch, max_targets, 2)),
                             rng.uniform(0.02, 0.5, (batch, max_targets, 2))], -1).astype(np.float32)
    mask = np.arange(max_targets)[None, :] < sizes[:, None]
    labels = np.where(mask, labels, 0).astype(np.int32)
    tboxes = np.where(mask[..., None], tboxes, 0.0).astype(np.float32)
    logits = rng.standard_normal((batch, queries, classes)).astype(np.float32)
    pboxes = np.concatenate([rng.uniform(0.05, 0.95, (batch, queries, 2)),
                             rng.uniform(0.02, 0.5, (batch, queries, 2))], -1).astype(np.float32)
    return logits, pboxes, labels, tboxes, mask, sizes

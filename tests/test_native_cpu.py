"""CPU-only checks of the native boundary: the library loads, exports every entry point the
header declares, and rejects bad arguments before touching a device.  No compute calls."""

from __future__ import annotations

import ctypes
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "rfdetr_b200.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(rfdetr_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_hot_path():
    names = _declared()
    for required in ("rfdetr_msda_forward", "rfdetr_msda_backward", "rfdetr_msda_backward_workspace_size",
                     "rfdetr_topk_select", "rfdetr_select_rows", "rfdetr_match_cost", "rfdetr_lsap_batched",
                     "rfdetr_status_string", "rfdetr_abi_version"):
        assert required in names


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg._native.lib()
    raw = ctypes.CDLL(pkg._native.LIB_PATH)
    for name in _declared():
        assert hasattr(raw, name), f"{name} declared in include/rfdetr_b200.h but not exported"
        assert name in pkg._native.SIGNATURES, f"{name} has no ctypes signature"
    assert lib.rfdetr_abi_version() == 3
    assert pkg._native.status_text(0) == "ok"
    assert "element type" in pkg._native.status_text(2)


def test_argument_validation_without_a_device(pkg):
    """Early-exit paths: invalid dtypes and shapes are reported before any CUDA call."""
    lib = pkg._native.lib()
    N = pkg._native
    shapes = N.int64_array([4, 4])
    # Unsupported dtype code.
    assert lib.rfdetr_msda_forward(None, None, 7, shapes, None, None, None, 0, None, 0, 1, 1, 4, 1, 1, 1) == N.ERR_DTYPE
    # Output dtype must be result_type(value, weights): bf16 x bf16 -> bf16.
    assert lib.rfdetr_msda_forward(None, None, 1, shapes, None, None, None, 1, None, 0, 1, 1, 4, 1, 1, 1) == N.ERR_DTYPE
    # Too many levels, negative sizes, inconsistent level_start_index.
    many = N.int64_array([2, 2] * 17)
    assert lib.rfdetr_msda_forward(None, None, 0, many, None, None, None, 0, None, 0, 1, 1, 4, 1, 17, 1) == N.ERR_SHAPE
    assert lib.rfdetr_msda_forward(None, None, 0, shapes, None, None, None, 0, None, 0, 1, -1, 4, 1, 1, 1) == N.ERR_SHAPE
    bad_start = N.int64_array([1])
    assert lib.rfdetr_msda_forward(None, None, 0, shapes, bad_start, None, None, 0, None, 0, 1, 1, 4, 1, 1,
                                   1) == N.ERR_SHAPE
    # Sizes whose element counts overflow int64 when multiplied are refused, not wrapped.
    huge = 1 << 40
    assert lib.rfdetr_msda_forward(None, None, 0, shapes, None, None, None, 0, None, 0, huge, huge, huge, huge, 1,
                                   1) == N.ERR_SHAPE
    assert lib.rfdetr_msda_forward(None, None, 0, shapes, None, None, None, 0, None, 0, 1 << 20, 1 << 20, 1 << 20,
                                   1, 1, 1) == N.ERR_SHAPE
    # Empty batch is a no-op.
    assert lib.rfdetr_msda_forward(None, None, 0, shapes, None, None, None, 0, None, 0, 0, 1, 4, 1, 1, 1) == N.OK
    assert lib.rfdetr_msda_backward_workspace_size(0, 8, 16, 16, 576) == 0
    assert lib.rfdetr_msda_backward_workspace_size(1, 8, 16, 16, 576) == 8 * 16 * 16 * 576 * 4
    # Top-k: k out of range, too many positions.
    assert lib.rfdetr_topk_select(None, None, 1, 10, 1, 11, None, None, None) == N.ERR_SHAPE
    assert lib.rfdetr_topk_select(None, None, 1, 20000, 2, 10, None, None, None) == N.ERR_SHAPE
    assert lib.rfdetr_topk_select(None, None, 1, 20000, 1, 4097, None, None, None) == N.ERR_SHAPE
    assert lib.rfdetr_topk_select(None, None, 1, (1 << 24) + 1, 1, 10, None, None, None) == N.ERR_SHAPE
    # Matcher: group count must divide the queries; target cap.
    assert lib.rfdetr_lsap_batched(None, None, None, 1, 10, 3, 3, None, None, None, None) == N.ERR_SHAPE
    assert lib.rfdetr_lsap_batched(None, None, None, 1, 10, 2000, 1, None, None, None, None) == N.ERR_SHAPE
    assert lib.rfdetr_match_cost(None, None, 5, None, 0, None, None, None, None, 1, 1, 1, 1, 2.0, 5.0, 2.0,
                                 0.25) == N.ERR_DTYPE


def test_python_api_rejects_cpu_tensors_and_unknown_names(pkg):
    value = torch.zeros((2, 4, 4))
    loc = torch.zeros((1, 3, 2, 1, 1, 2))
    attn = torch.zeros((1, 3, 2, 1))
    with pytest.raises(ValueError, match="unknown sampler"):
        pkg.ms_deform_attn_core_rows(value, ((2, 2),), loc, attn, "gather")
    with pytest.raises(ValueError, match="CUDA tensors"):
        pkg.ms_deform_attn_core_rows(value, ((2, 2),), loc, attn, "cuda")
    with pytest.raises(ValueError, match="unknown matcher"):
        pkg.CriterionConfig(matcher="auction").solve(torch.zeros((1, 4, 2)), torch.ones(1), 1)
    with pytest.raises(ValueError, match="CUDA tensors"):
        pkg.hungarian_match(torch.zeros((1, 4, 2)), torch.ones(1, dtype=torch.int32), 1)
    with pytest.raises(ValueError, match="CUDA tensors"):
        pkg.two_stage_topk(torch.zeros((2, 5, 3)), 2)


def test_tuning_knobs(pkg):
    """Knobs are set by name (no device needed); unknown names and malformed values are refused,
    and None restores the default."""
    N = pkg._native
    N.set_tuning("RFDETR_LSAP_STEP_CAP", "3")
    N.set_tuning("RFDETR_LSAP_STEP_CAP", None)
    N.set_tuning("RFDETR_MSDA_OWN", "24,1,0")
    N.set_tuning("RFDETR_MSDA_OWN", "")
    with pytest.raises(ValueError):
        N.set_tuning("RFDETR_NO_SUCH_KNOB", "1")
    with pytest.raises(ValueError):
        N.set_tuning("RFDETR_MSDA_OWN", "1,x")
    with pytest.raises(ValueError):
        N.set_tuning("RFDETR_MSDA_OWN", "1,2,3,4,5,6")


def test_ffi_sources_cover_every_entry_point():
    """The XLA FFI handlers (``rf-detr-jax_b200/ffi/rfdetr_ffi.cc``, not compiled here: JAX is
    absent) call every compute entry point the header declares, and the JAX module registers
    exactly the handlers the C++ file defines."""
    import ast

    ffi_dir = os.path.join(ROOT, "rf-detr-jax_b200", "ffi")
    cc = open(os.path.join(ffi_dir, "rfdetr_ffi.cc")).read()
    # The all-reduce replaces XLA's own collective (the train step's psum), not a custom call of
    # the model: it has no FFI handler.
    helpers = {"rfdetr_status_string", "rfdetr_abi_version", "rfdetr_set_tuning", "rfdetr_take_device_fault",
               "rfdetr_selftest_bounded_wait", "rfdetr_msda_backward_workspace_size", "rfdetr_ipc_handle_bytes",
               "rfdetr_allreduce_flag_bytes", "rfdetr_ipc_get_handle", "rfdetr_ipc_open_handle",
               "rfdetr_ipc_close_handle", "rfdetr_allreduce_sum_f32"}
    for name in _declared():
        if name not in helpers:
            assert re.search(rf"\b{name}\(", cc), f"{name} has no FFI handler"
    defined = set(re.findall(r"XLA_FFI_DEFINE_HANDLER_SYMBOL\((\w+),", cc))
    py = open(os.path.join(ffi_dir, "cuda_backend.py")).read()
    tree = ast.parse(py)
    handlers = None
    for node in ast.walk(tree):
        if isinstance(node, ast.Assign) and any(getattr(t, "id", None) == "HANDLERS" for t in node.targets):
            handlers = set(ast.literal_eval(node.value))
    assert handlers == defined
    called = set(re.findall(r'ffi_call\("(\w+)"', py))
    assert called <= defined and called >= defined - {"RfdetrMsdaBwdNoAlloc"}

"""The C-ABI library loads on a CPU-only machine, exports every declared entry
point, and rejects bad arguments before touching the GPU.

Mirrors the reference's export test (``tests/test_extension.py:17-40``) and the
ICHECK behaviour of ``csrc/ms_deformable_attn/ms_deform_attn_musa.mu:507-626``.
No call here launches a kernel: every case fails validation on the host.
"""

from __future__ import annotations

import ctypes
import re

import pytest
import torch

from conftest import ROOT
from muspace_b200.runtime import native

HEADER = ROOT / "include" / "muspace_msda.h"


def _declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"MSDA_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)


def test_header_declares_the_reference_entry_points():
    names = _declared_symbols()
    assert "ms_deform_attn_forward" in names
    assert "ms_deform_attn_backward" in names
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol():
    module = native.load_native_module()
    for name in _declared_symbols():
        assert hasattr(module.lib, name), name
    assert re.fullmatch(r"\d+\.\d+\.\d+", module.version())


def _inputs(dtype=torch.float32, batch=2, queries=3, heads=2, channels=4, levels=((2, 3), (1, 2)), points=2):
    lin = sum(h * w for h, w in levels)
    value = torch.zeros(batch, lin, heads, channels, dtype=dtype)
    shapes = torch.tensor(levels, dtype=torch.int64)
    start = torch.tensor([0, levels[0][0] * levels[0][1]], dtype=torch.int64)[: len(levels)]
    loc = torch.zeros(batch, queries, heads, len(levels), points, 2, dtype=dtype)
    weight = torch.zeros(batch, queries, heads, len(levels), points, dtype=dtype)
    out = torch.zeros(batch, queries, heads * channels, dtype=dtype)
    return [value, shapes, start, loc, weight, out]


def _forward(args, step=64):
    return native.native_function("ms_deform_attn_forward")(*args, step)


def test_cpu_tensors_are_rejected_before_any_launch():
    with pytest.raises(RuntimeError, match="value must be a CUDA tensor"):
        _forward(_inputs())


def test_float16_value_is_rejected_like_the_reference():
    with pytest.raises(RuntimeError, match="value must be float32 or bfloat16, got float16"):
        _forward(_inputs(torch.float16))


def test_backward_signature_is_bound_with_ten_arguments():
    fn = native.native_function("ms_deform_attn_backward")
    with pytest.raises(TypeError, match="takes 10 arguments"):
        fn(*_inputs())


def test_missing_export_is_explained():
    with pytest.raises(native.NativeModuleUnavailable, match="does not export 'missing_op'"):
        native.native_function("missing_op")


class _Dims(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in ("batch", "spatial_size", "heads", "channels", "levels", "queries", "points")]


def _plain_forward(dims, dtype=0):
    lib = native.load_native_module().lib
    lib.msda_forward.restype = ctypes.c_int
    lib.msda_forward.argtypes = [ctypes.c_int, ctypes.POINTER(_Dims)] + [ctypes.c_void_p] * 7
    return lib.msda_forward(dtype, ctypes.byref(dims), *([None] * 7))


def test_plain_pointer_entry_validates_sizes():
    module = native.load_native_module()
    assert _plain_forward(_Dims(1, 4, 1, 4, 1, 1, -1)) == 1
    assert "non-negative" in module.last_error()
    assert _plain_forward(_Dims(1, 4, 1, 4, 1, 1, 1), dtype=7) == 1
    assert "float32 or bfloat16" in module.last_error()
    # a non-empty problem with null pointers is refused on the host
    assert _plain_forward(_Dims(1, 4, 1, 4, 1, 1, 1)) == 1
    assert "null" in module.last_error()
    # an empty problem launches nothing and succeeds
    assert _plain_forward(_Dims(0, 4, 1, 4, 1, 1, 1)) == 0
    assert module.last_error() == ""


def test_static_scratch_backward_rejects_problems_beyond_its_array():
    """The no-allocation backward refuses, on the host and before any CUDA
    call, a problem whose work space exceeds its fixed array (c4: 3.84 M
    head-rows). The pointers are never touched on this path."""
    lib = native.load_native_module().lib
    fn = lib.msda_backward_static_scratch
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int, ctypes.POINTER(_Dims)] + [ctypes.c_void_p] * 10
    dims = _Dims(48, 30825, 8, 32, 4, 10000, 8)
    aligned = ctypes.c_void_p(256)  # never dereferenced: the size check fails first
    assert fn(1, ctypes.byref(dims), *([aligned] * 9), None) == 1
    assert "bytes of scratch" in native.load_native_module().last_error()


"""ctypes binding of the C oracle in ``msda_oracle.c`` -- TEST INFRASTRUCTURE ONLY.

The shared object is compiled with ``gcc`` into ``oracle/libmsda_oracle.so``
(git-ignored, rebuilt by :func:`build`). Arrays are numpy, row-major,
contiguous, with the layouts of ``mu_space/ops/multi_scale_deformable_attn.py:26-58``.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_SOURCE = _HERE / "msda_oracle.c"
_LIBRARY = _HERE / "libmsda_oracle.so"
_lib = None


class _Dims(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int64),
        ("spatial_size", ctypes.c_int64),
        ("heads", ctypes.c_int64),
        ("channels", ctypes.c_int64),
        ("levels", ctypes.c_int64),
        ("queries", ctypes.c_int64),
        ("points", ctypes.c_int64),
    ]


def build(force: bool = False) -> Path:
    """Compile the oracle with gcc (no fast-math, no FP contraction)."""
    if force or not _LIBRARY.exists() or _LIBRARY.stat().st_mtime < _SOURCE.stat().st_mtime:
        cmd = [
            "gcc",
            "-O2",
            "-std=c99",
            "-fPIC",
            "-shared",
            "-ffp-contract=off",
            "-fno-fast-math",
            str(_SOURCE),
            "-lm",
            "-o",
            str(_LIBRARY),
        ]
        subprocess.run(cmd, check=True)
    return _LIBRARY


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(_LIBRARY))
        ptr = ctypes.c_void_p
        lib.msda_oracle_forward.argtypes = [ctypes.POINTER(_Dims), ptr, ptr, ptr, ptr, ptr, ptr]
        lib.msda_oracle_forward.restype = None
        lib.msda_oracle_backward.argtypes = [ctypes.POINTER(_Dims)] + [ptr] * 9
        lib.msda_oracle_backward.restype = None
        _lib = lib
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _i64(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int64))


def _dims(value: np.ndarray, shapes: np.ndarray, loc: np.ndarray) -> _Dims:
    b, lin, heads, channels = value.shape
    _, queries, _, levels, points, _ = loc.shape
    if shapes.shape != (levels, 2):
        raise ValueError(f"spatial_shapes {shapes.shape} does not match {levels} levels")
    if int((shapes[:, 0] * shapes[:, 1]).sum()) != lin:
        raise ValueError("sum of H*W over levels must equal value.shape[1]")
    return _Dims(b, lin, heads, channels, levels, queries, points)


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def oracle_forward(value, spatial_shapes, level_start_index, sampling_locations, attention_weights):
    """Forward oracle: returns ``(B, Lq, Hh*D)`` float32."""
    value, loc, weight = _f32(value), _f32(sampling_locations), _f32(attention_weights)
    shapes, start = _i64(spatial_shapes), _i64(level_start_index)
    d = _dims(value, shapes, loc)
    out = np.zeros((d.batch, d.queries, d.heads * d.channels), dtype=np.float32)
    _load().msda_oracle_forward(
        ctypes.byref(d), _p(value), _p(shapes), _p(start), _p(loc), _p(weight), _p(out)
    )
    return out


def oracle_backward(
    value, spatial_shapes, level_start_index, sampling_locations, attention_weights, grad_output
):
    """Backward oracle: returns ``(grad_value, grad_loc, grad_weight)`` float32."""
    value, loc, weight = _f32(value), _f32(sampling_locations), _f32(attention_weights)
    shapes, start = _i64(spatial_shapes), _i64(level_start_index)
    d = _dims(value, shapes, loc)
    grad = _f32(grad_output).reshape(d.batch, d.queries, d.heads * d.channels)
    grad_value = np.zeros(value.shape, dtype=np.float64)
    grad_loc = np.zeros(loc.shape, dtype=np.float32)
    grad_weight = np.zeros(weight.shape, dtype=np.float32)
    _load().msda_oracle_backward(
        ctypes.byref(d),
        _p(value),
        _p(shapes),
        _p(start),
        _p(loc),
        _p(weight),
        _p(grad),
        _p(grad_value),
        _p(grad_loc),
        _p(grad_weight),
    )
    return grad_value.astype(np.float32), grad_loc, grad_weight

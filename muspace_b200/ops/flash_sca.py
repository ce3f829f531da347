"""FlashSCA (``flash_bevpool_sca``), B200 build.

Drop-in for the spatial-cross-attention half of ``mu_space/ops/flashbev.py``
(``flash_bevpool_sca``, 560-684; autograd ``_FlashSCAModule``, 457-557): same
signature and keyword arguments (``grid_size`` with either ``voxel_size`` +
``voxel_min`` or ``roi_range``, ``num_heads``, ``num_points``,
``value_stride_n``, ``epsilon``, ``backend``), the same validation messages,
and gradients for value, sampling offsets and attention weights. The
reference's ``_sanitize_value`` pass (non-finite values to 0, with a host
sync) happens inside the kernels' gathers instead.

What differs, on purpose: the work runs in the sm_100a kernels of
``libmuspace_ops.so`` only; CPU tensors, ``backend="reference"`` and a failing
native library raise instead of falling back to the reference's Python loop.
"""

from __future__ import annotations

from typing import Sequence

import torch

from ..runtime.kernel_dispatch import (
    DispatchDecision,
    DispatchReport,
    explain_dispatch as _explain_dispatch,
    record_dispatch_report,
)
from ..runtime.native import NativeModuleUnavailable, native_module_proxy

SCA_OPERATOR_NAME = "flash_bevpool_sca"


def _native_extension():
    try:
        return native_module_proxy()
    except NativeModuleUnavailable:
        return None


def _triple(values: Sequence[float], name: str) -> tuple[float, float, float]:
    if len(values) != 3:
        raise ValueError(f"{name} must contain three values")
    return tuple(float(v) for v in values)  # type: ignore[return-value]


def _grid(values: Sequence[int]) -> tuple[int, int, int]:
    if len(values) != 3:
        raise ValueError("grid_size must contain [x, y, z]")
    result = tuple(int(v) for v in values)
    if any(v <= 0 for v in result):
        raise ValueError("grid_size values must be positive")
    return result  # type: ignore[return-value]


def _check_float(tensor: torch.Tensor, name: str) -> None:
    if tensor.dtype != torch.float32:
        raise TypeError(f"{name} must use float32")
    if not tensor.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _check_int(tensor: torch.Tensor, name: str) -> None:
    if tensor.dtype != torch.int32:
        raise TypeError(f"{name} must use int32")


def _resolve_voxels(grid_size, voxel_size, voxel_min, roi_range):
    """Reference ``flashbev.py:264-286``: (grid, (sx, sy, sz, xmin, ymin, zmin))."""
    grid = _grid(grid_size)
    if roi_range is not None:
        if voxel_size is not None or voxel_min is not None:
            raise ValueError("pass either roi_range or voxel_size/voxel_min")
        if len(roi_range) != 6:
            raise ValueError("roi_range must contain [xmin,xmax,ymin,ymax,zmin,zmax]")
        values = ([float(v) for v in roi_range.detach().cpu().tolist()] if isinstance(roi_range, torch.Tensor)
                  else [float(v) for v in roi_range])
        return grid, ((values[1] - values[0]) / grid[0], (values[3] - values[2]) / grid[1],
                      (values[5] - values[4]) / grid[2], values[0], values[2], values[4])
    if voxel_size is None or voxel_min is None:
        raise ValueError("voxel_size and voxel_min are required when roi_range is absent")
    return grid, _triple(voxel_size, "voxel_size") + _triple(voxel_min, "voxel_min")


class _FlashSCAFunction(torch.autograd.Function):
    """Autograd over ``flash_bevpool_sca_{forward,backward}`` (reference 457-557):
    the backward zero-fills the three gradient buffers the kernel accumulates
    into and passes the voxel grid as the reference's 6-float roi tensor."""

    @staticmethod
    def forward(ctx, value, projections, spatial_shapes, level_start, image_size, offsets, weights, num_heads,
                num_points, grid, voxel, value_stride_n, epsilon):
        ext = _native_extension()
        if ext is None:
            raise RuntimeError("muSPACE-B200 native library is unavailable")
        gx, gy, gz = grid
        sx, sy, sz, xmin, ymin, zmin = voxel
        output = value.new_empty((value.size(0), gy, gx, value.size(3)))
        ext.flash_bevpool_sca_forward(value, projections, spatial_shapes, level_start, image_size, offsets, weights,
                                      output, num_heads, num_points, gx, gy, gz, sx, sy, sz, xmin, ymin, zmin,
                                      value_stride_n, epsilon)
        roi = value.new_tensor([xmin, xmin + gx * sx, ymin, ymin + gy * sy, zmin, zmin + gz * sz])
        ctx.save_for_backward(value, projections, spatial_shapes, level_start, image_size, roi, offsets, weights)
        ctx.params = (num_heads, num_points, grid, value_stride_n, epsilon)
        return output

    @staticmethod
    def backward(ctx, grad_output):
        value, projections, spatial_shapes, level_start, image_size, roi, offsets, weights = ctx.saved_tensors
        num_heads, num_points, (gx, gy, gz), stride, epsilon = ctx.params
        ext = _native_extension()
        if ext is None:
            raise RuntimeError("muSPACE-B200 native library is unavailable")
        grad_value = torch.zeros_like(value)
        grad_offsets = torch.zeros_like(offsets)
        grad_weights = torch.zeros_like(weights)
        ext.flash_bevpool_sca_backward(grad_output.contiguous(), value, projections, spatial_shapes, level_start,
                                       image_size, roi, offsets, weights, grad_value, grad_offsets, grad_weights,
                                       num_heads, num_points, gx, gy, gz, stride, epsilon)
        return (grad_value, None, None, None, None, grad_offsets, grad_weights, None, None, None, None, None, None)


def _report(backend: str, decision: DispatchDecision, selected: str, reason: str, native_available: bool):
    record_dispatch_report(DispatchReport(operator=SCA_OPERATOR_NAME, requested_backend=backend,
                                          selected_backend=selected, device=decision.device, reason=reason,
                                          native_available=native_available))


def flash_bevpool_sca(value, projection_matrices, spatial_shapes, level_start_index, image_size, sampling_offsets,
                      attention_weights, grid_size, voxel_size=None, voxel_min=None, *, roi_range=None,
                      num_heads=None, num_points=None, value_stride_n=None, epsilon=1e-5, backend: str = "auto"):
    """BEV features ``[B, gy, gx, C]`` from multi-camera features ``value [B, N, S, C]``.

    projection_matrices ``[B, N, 3, 4]``; spatial_shapes ``[L, 2]`` / level_start_index
    ``[L]`` / image_size ``[2]`` int32; sampling_offsets ``[B, gy, gx, heads, L, P,
    gz, 2]`` and attention_weights ``[B, gy, gx, heads, L, P, gz]`` float32.
    """
    for tensor, name in ((value, "value"), (projection_matrices, "projection_matrices"),
                         (sampling_offsets, "sampling_offsets"), (attention_weights, "attention_weights")):
        _check_float(tensor, name)
    for tensor, name in ((spatial_shapes, "spatial_shapes"), (level_start_index, "level_start_index"),
                         (image_size, "image_size")):
        _check_int(tensor, name)
    if value.dim() != 4 or sampling_offsets.dim() != 8 or attention_weights.dim() != 7:
        raise ValueError("invalid FlashSCA input ranks")
    heads = int(num_heads or sampling_offsets.size(3))
    points = int(num_points or sampling_offsets.size(5))
    if heads <= 0 or points <= 0:
        raise ValueError("num_heads and num_points must be positive")
    if value.size(3) % heads != 0:
        raise ValueError("channels must be divisible by num_heads")
    grid, voxel = _resolve_voxels(grid_size, voxel_size, voxel_min, roi_range)
    gx, gy, gz = grid
    if projection_matrices.shape != (value.size(0), value.size(1), 3, 4):
        raise ValueError("projection_matrices must have shape [B,N,3,4]")
    if spatial_shapes.dim() != 2 or spatial_shapes.size(1) != 2:
        raise ValueError("spatial_shapes must have shape [levels,2]")
    levels = spatial_shapes.size(0)
    if level_start_index.shape != (levels,) or image_size.numel() != 2:
        raise ValueError("level_start_index/image_size shapes must be [levels]/[2]")
    expected_offsets = (value.size(0), gy, gx, heads, levels, points, gz, 2)
    if tuple(sampling_offsets.shape) != expected_offsets:
        raise ValueError(f"sampling_offsets must have shape {expected_offsets}")
    if tuple(attention_weights.shape) != expected_offsets[:-1]:
        raise ValueError(f"attention_weights must have shape {expected_offsets[:-1]}")
    stride = int(value_stride_n or value.size(2))
    if stride <= 0 or stride > value.size(2):
        raise ValueError("value_stride_n must be in [1, value.size(2)]")
    native_available = _native_extension() is not None
    decision = _explain_dispatch(value, backend=backend, native_available=native_available,
                                 operator=SCA_OPERATOR_NAME)
    if decision.backend == "error":
        _report(backend, decision, "error", decision.reason, native_available)
        raise RuntimeError(decision.reason)
    device = value.device
    spatial_shapes, level_start_index, image_size = (t.to(device).contiguous() for t in
                                                     (spatial_shapes, level_start_index, image_size))
    level_ends = level_start_index + spatial_shapes[:, 0] * spatial_shapes[:, 1]
    if bool((spatial_shapes <= 0).any()) or bool((level_start_index < 0).any()) or bool((level_ends > stride).any()):
        raise ValueError("value_stride_n must cover every positive spatial level")
    try:
        result = _FlashSCAFunction.apply(value, projection_matrices.contiguous(), spatial_shapes, level_start_index,
                                         image_size, sampling_offsets, attention_weights, heads, points, grid, voxel,
                                         stride, float(epsilon))
    except RuntimeError as exc:
        _report(backend, decision, "error", str(exc), native_available)
        raise
    _report(backend, decision, "cuda", decision.reason, native_available)
    return result


__all__ = ["flash_bevpool_sca"]

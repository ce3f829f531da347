"""SparseDrive deformable aggregation, B200 build.

Drop-in for ``mu_space/ops/deformable_aggregation.py`` of the reference:
``deformable_aggregation`` keeps its signature (``backend=``), its input
validation and error messages (float32 features / locations / weights, int32
shape tables, ranks, ``1 <= groups <= 8``, ``C % groups == 0``), its zero-anchor
short circuit, its autograd Function over the ``*_opt`` native pair, its
dispatch report, and the SparseDrive helpers ``deformable_aggregation_function``
and ``feature_maps_format``.

What differs, on purpose: the work runs in the sm_100a kernels of
``libmuspace_ops.so`` only. CPU tensors, ``backend="reference"`` and a missing
or failing native library raise instead of falling back to a CPU path, and
the reference's pure-Python ``deformable_aggregation_reference`` is not part of
the build.
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

OPERATOR_NAME = "deformable_aggregation"
MAX_GROUPS = 8


def _native_extension():
    try:
        return native_module_proxy()
    except NativeModuleUnavailable:
        return None


def _normalize_inputs(mc_ms_feat, spatial_shape, scale_start_index, sampling_location, weights):
    """Reference ``ops/deformable_aggregation.py:35-79``; additionally brings the
    int32 tables to the features' CUDA device when they were left on the host."""
    if mc_ms_feat.dtype != torch.float32:
        raise TypeError("mc_ms_feat must use float32")
    if sampling_location.dtype != torch.float32:
        raise TypeError("sampling_location must use float32")
    if weights.dtype != torch.float32:
        raise TypeError("weights must use float32")
    if spatial_shape.dtype != torch.int32:
        raise TypeError("spatial_shape must use int32")
    if scale_start_index.dtype != torch.int32:
        raise TypeError("scale_start_index must use int32")
    if mc_ms_feat.dim() != 3:
        raise ValueError("mc_ms_feat must have shape [B, num_feat, C]")
    if spatial_shape.dim() != 3 or spatial_shape.size(-1) != 2:
        raise ValueError("spatial_shape must have shape [num_cams, num_scale, 2]")
    if scale_start_index.dim() != 2:
        raise ValueError("scale_start_index must have shape [num_cams, num_scale]")
    if sampling_location.dim() != 5 or sampling_location.size(-1) != 2:
        raise ValueError("sampling_location must have shape [B, anchors, pts, cams, 2]")
    if weights.dim() != 6:
        raise ValueError("weights must have shape [B, anchors, pts, cams, scale, groups]")
    num_embeds, num_groups = mc_ms_feat.size(-1), weights.size(-1)
    if num_groups <= 0 or num_groups > MAX_GROUPS:
        raise ValueError(f"num_groups must be in [1, {MAX_GROUPS}]")
    if num_embeds % num_groups != 0:
        raise ValueError("num_embeds must be divisible by num_groups")
    if mc_ms_feat.device.type == "cuda":
        spatial_shape = spatial_shape.to(mc_ms_feat.device)
        scale_start_index = scale_start_index.to(mc_ms_feat.device)
    return tuple(t.contiguous() for t in (mc_ms_feat, spatial_shape, scale_start_index, sampling_location, weights))


class _NativeDeformableAggregationFunction(torch.autograd.Function):
    """Autograd over ``deformable_aggregation_{forward,backward}_opt``
    (reference ``ops/deformable_aggregation.py:159-213``). The backward zeroes
    ``grad_mc_ms_feat`` (the kernel accumulates into it); the kernel writes every
    element of the location and weight gradients."""

    @staticmethod
    def forward(ctx, mc_ms_feat, spatial_shape, scale_start_index, sampling_location, weights):
        ext = _native_extension()
        if ext is None:
            raise RuntimeError("muSPACE-B200 native library is unavailable")
        output = mc_ms_feat.new_empty((mc_ms_feat.size(0), sampling_location.size(1), mc_ms_feat.size(2)))
        ext.deformable_aggregation_forward_opt(mc_ms_feat, spatial_shape, scale_start_index, sampling_location,
                                               weights, output)
        ctx.save_for_backward(mc_ms_feat, spatial_shape, scale_start_index, sampling_location, weights)
        return output

    @staticmethod
    def backward(ctx, grad_output):
        ext = _native_extension()
        if ext is None:
            raise RuntimeError("muSPACE-B200 native library is unavailable")
        mc_ms_feat, spatial_shape, scale_start_index, sampling_location, weights = ctx.saved_tensors
        grad_mc_ms_feat = torch.zeros_like(mc_ms_feat)
        grad_sampling_location = torch.empty_like(sampling_location)
        grad_weights = torch.empty_like(weights)
        ext.deformable_aggregation_backward_opt(mc_ms_feat, spatial_shape, scale_start_index, sampling_location,
                                                weights, grad_output.contiguous(), grad_mc_ms_feat,
                                                grad_sampling_location, grad_weights)
        return grad_mc_ms_feat, None, None, grad_sampling_location, grad_weights


def _report(backend: str, decision: DispatchDecision, selected: str, reason: str, native_available: bool):
    record_dispatch_report(
        DispatchReport(
            operator=OPERATOR_NAME,
            requested_backend=backend,
            selected_backend=selected,
            device=decision.device,
            reason=reason,
            native_available=native_available,
        )
    )


def deformable_aggregation(mc_ms_feat: torch.Tensor, spatial_shape: torch.Tensor, scale_start_index: torch.Tensor,
                           sampling_location: torch.Tensor, weights: torch.Tensor, *,
                           backend: str = "auto") -> torch.Tensor:
    """Multi-camera multi-scale deformable aggregation (differentiable).

    mc_ms_feat ``[B, num_feat, C]``; spatial_shape ``[cams, scales, 2]`` int32
    (H, W); scale_start_index ``[cams, scales]`` int32; sampling_location
    ``[B, anchors, pts, cams, 2]`` (x, y); weights ``[B, anchors, pts, cams,
    scales, groups]``. Returns ``[B, anchors, C]``.
    """
    mc_ms_feat, spatial_shape, scale_start_index, sampling_location, weights = _normalize_inputs(
        mc_ms_feat, spatial_shape, scale_start_index, sampling_location, weights)
    native_available = _native_extension() is not None
    decision = _explain_dispatch(mc_ms_feat, backend=backend, native_available=native_available,
                                 operator=OPERATOR_NAME)
    if decision.backend == "error":
        _report(backend, decision, "error", decision.reason, native_available)
        raise RuntimeError(decision.reason)
    for name, tensor in (("sampling_location", sampling_location), ("weights", weights)):
        if tensor.device != mc_ms_feat.device:
            reason = f"{name} is on {tensor.device}, mc_ms_feat is on {mc_ms_feat.device}"
            _report(backend, decision, "error", reason, native_available)
            raise RuntimeError(reason)
    if sampling_location.size(1) == 0:
        _report(backend, decision, "cuda", decision.reason, native_available)
        output = mc_ms_feat.new_zeros((mc_ms_feat.size(0), 0, mc_ms_feat.size(2)))
        return output + mc_ms_feat.sum() * 0 + sampling_location.sum() * 0 + weights.sum() * 0
    try:
        output = _NativeDeformableAggregationFunction.apply(mc_ms_feat, spatial_shape, scale_start_index,
                                                            sampling_location, weights)
    except RuntimeError as exc:
        _report(backend, decision, "error", str(exc), native_available)
        raise
    _report(backend, decision, "cuda", decision.reason, native_available)
    return output


def deformable_aggregation_function(feature_maps: torch.Tensor, spatial_shape: torch.Tensor,
                                    scale_start_index: torch.Tensor, sampling_location: torch.Tensor,
                                    weights: torch.Tensor, *, backend: str = "auto") -> torch.Tensor:
    """SparseDrive-compatible alias: casts to the op's dtypes first
    (reference ``ops/deformable_aggregation.py:320-337``)."""
    return deformable_aggregation(
        feature_maps.contiguous().float(),
        spatial_shape.contiguous().to(dtype=torch.int32),
        scale_start_index.contiguous().to(dtype=torch.int32),
        sampling_location.contiguous().float(),
        weights.contiguous().float(),
        backend=backend,
    )


def feature_maps_format(feature_maps, inverse: bool = False):
    """SparseDrive's packing of per-level camera feature maps (reference
    ``ops/deformable_aggregation.py:340-425``).

    Forward: a list of levels ``[B, cams, C, H_l, W_l]`` (or a list of such
    lists, concatenated along the feature rows) becomes
    ``[col_feats [B, cams * sum(H_l W_l), C], spatial_shape [cams, L, 2] int64,
    scale_start_index [cams, L] int64]``, camera-major, level-minor.
    ``inverse=True`` undoes it, returning per run of cameras with equal shapes
    the list of levels ``[B, cams_in_run, C, H_l, W_l]``.
    """
    if inverse:
        col_feats, spatial_shape, _scale_start_index = feature_maps
        sizes = (spatial_shape[..., 0] * spatial_shape[..., 1]).tolist()
        shapes = spatial_shape.tolist()
        runs: list[list[int]] = []  # consecutive cameras with identical level shapes
        for cam in range(len(shapes)):
            if runs and shapes[cam] == shapes[runs[-1][0]]:
                runs[-1].append(cam)
            else:
                runs.append([cam])
        out, row = [], 0
        for cams in runs:
            per_cam = sum(sizes[cams[0]])
            block = col_feats[:, row:row + per_cam * len(cams)].unflatten(1, (len(cams), per_cam))
            row += per_cam * len(cams)
            levels, offset = [], 0
            for (h, w), size in zip(shapes[cams[0]], sizes[cams[0]]):
                level = block[:, :, offset:offset + size].unflatten(2, (int(h), int(w)))
                levels.append(level.permute(0, 1, 4, 2, 3))
                offset += size
            out.append(levels)
        return out

    if isinstance(feature_maps[0], (list, tuple)):
        parts = [feature_maps_format(x) for x in feature_maps]
        return [torch.cat([p[0] for p in parts], dim=1), torch.cat([p[1] for p in parts], dim=0),
                torch.cat([p[2] for p in parts], dim=0)]

    batch, cams = feature_maps[0].shape[:2]
    shapes: list[Sequence[int]] = [tuple(f.shape[-2:]) for f in feature_maps]
    # [B, cams, C, H, W] -> [B, cams, H*W, C], levels side by side, cameras stacked
    col = torch.cat([f.flatten(3).transpose(2, 3) for f in feature_maps], dim=2).flatten(1, 2)
    spatial_shape = torch.tensor([shapes] * cams, dtype=torch.int64, device=col.device)
    sizes = (spatial_shape[..., 0] * spatial_shape[..., 1]).flatten()
    starts = torch.cat([sizes.new_zeros(1), sizes.cumsum(0)[:-1]]).view(cams, -1)
    return [col, spatial_shape, starts]


def explain_dispatch(mc_ms_feat: torch.Tensor, *, backend: str = "auto") -> DispatchDecision:
    return _explain_dispatch(mc_ms_feat, backend=backend, native_available=_native_extension() is not None,
                             operator=OPERATOR_NAME)


__all__ = [
    "deformable_aggregation",
    "deformable_aggregation_function",
    "explain_dispatch",
    "feature_maps_format",
]

"""Canonical multi-scale deformable attention op, B200 build.

Drop-in for ``mu_space/ops/multi_scale_deformable_attn.py`` of the reference:
``multi_scale_deformable_attn`` keeps its signature (``im2col_step=64``,
``backend=``), its input normalisation (int64 shape tensors, float16 /
bfloat16 / float32 values, locations and weights cast to the value dtype,
contiguous views), its zero-query short circuit, its autograd Function with
the same six-gradient contract and dtype handling, its dispatch report, and
the mmcv four-argument wrapper ``multi_scale_deformable_attn_pytorch_compat``.

What differs, on purpose: the work runs in the sm_100a kernels of
``libmuspace_ops.so`` only. CPU tensors, ``backend="reference"`` and a missing
or failing native library raise instead of falling back to a CPU path.
"""

from __future__ import annotations

import torch

from ..runtime.kernel_dispatch import (
    DispatchDecision,
    DispatchReport,
    explain_dispatch as _explain_dispatch,
    record_dispatch_report,
)
from ..runtime.native import NativeModuleUnavailable, native_module_proxy

OPERATOR_NAME = "multi_scale_deformable_attn"


def _native_extension():
    try:
        return native_module_proxy()
    except NativeModuleUnavailable:
        return None


def _level_start_index(spatial_shapes: torch.Tensor) -> torch.Tensor:
    level_sizes = spatial_shapes[:, 0] * spatial_shapes[:, 1]
    return torch.cat([level_sizes.new_zeros(1), level_sizes.cumsum(0)[:-1]])


def multi_scale_deformable_attn_pytorch_compat(
    value: torch.Tensor,
    value_spatial_shapes: torch.Tensor,
    sampling_locations: torch.Tensor,
    attention_weights: torch.Tensor,
) -> torch.Tensor:
    """mmcv's four-argument signature; derives ``level_start_index`` by cumsum
    (reference ``ops/multi_scale_deformable_attn.py:61-75``)."""
    return multi_scale_deformable_attn(
        value,
        value_spatial_shapes,
        _level_start_index(value_spatial_shapes),
        sampling_locations,
        attention_weights,
    )


def _to_contiguous(*tensors: torch.Tensor) -> tuple[torch.Tensor, ...]:
    return tuple(t.contiguous() for t in tensors)


def _requires_native_backend(
    value: torch.Tensor,
    spatial_shapes: torch.Tensor,
    level_start_index: torch.Tensor,
    sampling_locations: torch.Tensor,
    attention_weights: torch.Tensor,
) -> bool:
    return any(
        t.device.type == "cuda"
        for t in (value, spatial_shapes, level_start_index, sampling_locations, attention_weights)
    )


def deterministic_workspace_bytes(value: torch.Tensor, sampling_locations: torch.Tensor) -> int:
    """Work space of the deterministic backward for these views, as the
    library computes it (``msda_deterministic_workspace_bytes``)."""
    from ..runtime.native import deterministic_workspace_bytes as query

    batch, spatial, heads, channels = value.shape
    _, queries, _, levels, points, _ = sampling_locations.shape
    return query(batch, spatial, heads, channels, levels, queries, points)


class _NativeMSDAFunction(torch.autograd.Function):
    """Autograd over the two C-ABI calls (reference ``ops/...:101-190``).

    bfloat16 reaches the kernels as bfloat16; float16 and float32 are computed
    from fp32 storage and cast back. The backward hands the kernel fp32
    gradient buffers: ``grad_value`` zero-filled (the kernel accumulates into
    it), ``grad_sampling`` / ``grad_attention`` uninitialised because the
    kernel writes every element of them. Under
    ``torch.use_deterministic_algorithms(True)`` the backward runs the
    deterministic entry point (bit-identical ``grad_value`` from run to run).
    """

    @staticmethod
    def forward(
        ctx,
        value: torch.Tensor,
        spatial_shapes: torch.Tensor,
        level_start_index: torch.Tensor,
        sampling_locations: torch.Tensor,
        attention_weights: torch.Tensor,
        im2col_step: int,
    ) -> torch.Tensor:
        ext = _native_extension()
        if ext is None:
            raise RuntimeError("muSPACE-B200 native library is unavailable")
        ctx.im2col_step = im2col_step
        ctx.value_dtype = value.dtype
        ctx.sampling_dtype = sampling_locations.dtype
        ctx.attention_dtype = attention_weights.dtype
        if value.dtype == torch.bfloat16:
            value_arg, sampling_arg, attn_arg = _to_contiguous(value, sampling_locations, attention_weights)
        else:
            value_arg, sampling_arg, attn_arg = _to_contiguous(
                value.float(), sampling_locations.float(), attention_weights.float()
            )
        spatial_shapes = spatial_shapes.contiguous()
        level_start_index = level_start_index.contiguous()
        output = value_arg.new_empty(
            (value_arg.size(0), sampling_arg.size(1), value_arg.size(2) * value_arg.size(3))
        )
        ext.ms_deform_attn_forward(
            value_arg, spatial_shapes, level_start_index, sampling_arg, attn_arg, output, im2col_step
        )
        ctx.save_for_backward(value_arg, spatial_shapes, level_start_index, sampling_arg, attn_arg)
        return output.to(dtype=ctx.value_dtype)

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor) -> tuple[torch.Tensor | None, ...]:
        ext = _native_extension()
        if ext is None:
            raise RuntimeError("muSPACE-B200 native library is unavailable")
        value, spatial_shapes, level_start_index, sampling_locations, attention_weights = ctx.saved_tensors
        grad_value = torch.zeros_like(value, dtype=torch.float32)
        grad_sampling = torch.empty_like(sampling_locations, dtype=torch.float32)
        grad_attention = torch.empty_like(attention_weights, dtype=torch.float32)
        grad_output = grad_output.to(dtype=value.dtype).contiguous()
        args = (value, spatial_shapes, level_start_index, sampling_locations, attention_weights, grad_output,
                grad_value, grad_sampling, grad_attention)
        if torch.are_deterministic_algorithms_enabled():
            # reproducible grad_value: 64-bit fixed-point sums on a work space
            workspace = torch.empty(deterministic_workspace_bytes(value, sampling_locations), dtype=torch.uint8,
                                    device=value.device)
            ext.ms_deform_attn_backward_deterministic(*args, workspace, ctx.im2col_step)
        else:
            ext.ms_deform_attn_backward(*args, ctx.im2col_step)
        return (
            grad_value.to(dtype=ctx.value_dtype),
            None,
            None,
            grad_sampling.to(dtype=ctx.sampling_dtype),
            grad_attention.to(dtype=ctx.attention_dtype),
            None,
        )


def _normalize_inputs(
    value: torch.Tensor,
    spatial_shapes: torch.Tensor,
    level_start_index: torch.Tensor,
    sampling_locations: torch.Tensor,
    attention_weights: torch.Tensor,
) -> tuple[torch.Tensor, ...]:
    """Reference ``ops/...:193-212``; additionally brings the two small int64
    tables to the value's CUDA device when they were left on the host."""
    if spatial_shapes.dtype != torch.int64:
        raise TypeError("spatial_shapes must be int64")
    if level_start_index.dtype != torch.int64:
        raise TypeError("level_start_index must be int64")
    if value.dtype not in {torch.float16, torch.bfloat16, torch.float32}:
        raise TypeError("value must be float16, bfloat16 or float32")
    if sampling_locations.dtype != value.dtype:
        sampling_locations = sampling_locations.to(dtype=value.dtype)
    if attention_weights.dtype != value.dtype:
        attention_weights = attention_weights.to(dtype=value.dtype)
    if value.device.type == "cuda":
        spatial_shapes = spatial_shapes.to(value.device)
        level_start_index = level_start_index.to(value.device)
    return _to_contiguous(value, spatial_shapes, level_start_index, sampling_locations, attention_weights)


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


def multi_scale_deformable_attn(
    value: torch.Tensor,
    spatial_shapes: torch.Tensor,
    level_start_index: torch.Tensor,
    sampling_locations: torch.Tensor,
    attention_weights: torch.Tensor,
    *,
    im2col_step: int = 64,
    backend: str = "auto",
) -> torch.Tensor:
    """MSDA forward (differentiable): ``(B, Lq, Hh*D)`` output in ``value.dtype``.

    value ``(B, Lin, Hh, D)``; spatial_shapes ``(L, 2)`` int64 as (H, W);
    level_start_index ``(L,)`` int64; sampling_locations ``(B, Lq, Hh, L, P, 2)``
    as (x, y) in [0, 1]; attention_weights ``(B, Lq, Hh, L, P)``. Bilinear
    sampling with zero padding, ``align_corners=False`` (grid_sample's rules).
    """
    value, spatial_shapes, level_start_index, sampling_locations, attention_weights = _normalize_inputs(
        value, spatial_shapes, level_start_index, sampling_locations, attention_weights
    )
    native_available = _native_extension() is not None
    decision = _explain_dispatch(value, backend=backend, native_available=native_available)
    if decision.backend == "error":
        _report(backend, decision, "error", decision.reason, native_available)
        raise RuntimeError(decision.reason)
    for name, tensor in (("sampling_locations", sampling_locations), ("attention_weights", attention_weights)):
        if tensor.device != value.device:
            reason = f"{name} is on {tensor.device}, value is on {value.device}"
            _report(backend, decision, "error", reason, native_available)
            raise RuntimeError(reason)
    if sampling_locations.size(1) == 0:
        output = value.new_zeros((value.size(0), 0, value.size(2) * value.size(3)))
        _report(backend, decision, "cuda", decision.reason, native_available)
        # keep every input in the graph so their gradients are defined (zeros)
        return output + value.sum() * 0 + sampling_locations.sum() * 0 + attention_weights.sum() * 0
    try:
        output = _NativeMSDAFunction.apply(
            value, spatial_shapes, level_start_index, sampling_locations, attention_weights, im2col_step
        )
    except RuntimeError as exc:
        _report(backend, decision, "error", str(exc), native_available)
        raise
    _report(backend, decision, "cuda", decision.reason, native_available)
    return output


def explain_dispatch(value: torch.Tensor, *, backend: str = "auto") -> DispatchDecision:
    return _explain_dispatch(value, backend=backend, native_available=_native_extension() is not None)

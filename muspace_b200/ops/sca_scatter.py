"""BEVFormer spatial cross-attention: MSDA forward fused with the rebatch
scatter and the camera-count normalisation.

BEVFormer's ``SpatialCrossAttention`` rebatches the BEV queries that each camera
sees into ``(B * cams, max_len, ...)`` tensors, runs MSDA on them, then adds
every camera's output rows back into the BEV ``slots`` at ``index`` and divides
by the number of cameras that saw each BEV query. The reference fused the last
two steps into its forward kernel
(``ms_deformable_im2col_scatter_div_musa``,
``csrc/ms_deformable_attn/ms_deform_attn_musa.mu:455-505``; kernel
``ms_deform_attn_musa_kernel.muh:419-486``) but never exported it. Here it is
the C-ABI export ``ms_deform_attn_scatter_div_forward`` (one camera per call,
the reference's contract), wrapped by:

* :func:`ms_deform_attn_scatter_div` -- one camera, ``slots`` updated in place;
* :func:`sca_rebatch_scatter` -- all cameras in order (one launch each).

Forward only, as in the reference: the fused step serves inference; training
keeps the unfused MSDA op and its autograd.
"""

from __future__ import annotations

from typing import Sequence

import torch

from ..runtime.native import native_function

_STORAGE = (torch.float32, torch.bfloat16)


def _check(value, spatial_shapes, level_start_index, sampling_locations, attention_weights, index, count, slots):
    tensors = {
        "value": value, "spatial_shapes": spatial_shapes, "level_start_index": level_start_index,
        "sampling_locations": sampling_locations, "attention_weights": attention_weights, "index": index,
        "count": count, "slots": slots,
    }
    for name, t in tensors.items():
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a tensor")
        if t.device.type != "cuda":
            raise RuntimeError(f"{name} must be a CUDA tensor (the fused scatter has no CPU path)")
    if value.dtype not in _STORAGE:
        raise TypeError("value must be float32 or bfloat16")
    for name in ("sampling_locations", "attention_weights", "count", "slots"):
        if tensors[name].dtype != value.dtype:
            raise TypeError(f"{name} must have the dtype of value ({value.dtype})")
    for name in ("spatial_shapes", "level_start_index", "index"):
        if tensors[name].dtype != torch.int64:
            raise TypeError(f"{name} must be int64")
    if not slots.is_contiguous():
        raise ValueError("slots must be contiguous (it is updated in place)")


def ms_deform_attn_scatter_div(value: torch.Tensor, spatial_shapes: torch.Tensor, level_start_index: torch.Tensor,
                               sampling_locations: torch.Tensor, attention_weights: torch.Tensor,
                               index: torch.Tensor, count: torch.Tensor, slots: torch.Tensor,
                               cam_id: int) -> torch.Tensor:
    """``slots[b, index[q]] += MSDA(b * cams + cam_id, q) / count[b, index[q]]`` for one camera.

    value ``(B * cams, Lin, Hh, D)``; sampling_locations ``(B * cams, max_len,
    Hh, L, P, 2)`` and attention_weights ``(B * cams, max_len, Hh, L, P)`` hold
    the rebatched queries; index ``(valid_len,)`` int64 holds the distinct BEV
    queries of this camera's first ``valid_len`` rows; count ``(B, num_query)``
    and slots ``(B, num_query, Hh * D)`` share value's dtype. Returns ``slots``.
    """
    _check(value, spatial_shapes, level_start_index, sampling_locations, attention_weights, index, count, slots)
    native_function("ms_deform_attn_scatter_div_forward")(
        value.contiguous(), spatial_shapes.contiguous(), level_start_index.contiguous(),
        sampling_locations.contiguous(), attention_weights.contiguous(), index.contiguous(), count.contiguous(),
        slots, int(cam_id))
    return slots


def sca_rebatch_scatter(value: torch.Tensor, spatial_shapes: torch.Tensor, level_start_index: torch.Tensor,
                        sampling_locations: torch.Tensor, attention_weights: torch.Tensor,
                        indexes: Sequence[torch.Tensor], count: torch.Tensor,
                        slots: torch.Tensor | None = None) -> torch.Tensor:
    """All cameras: the SCA output ``sum_cam scatter(MSDA_cam) / count``.

    ``indexes[cam]`` lists camera ``cam``'s BEV queries (BEVFormer's
    ``bev_mask[cam].sum(-1).nonzero()``); ``slots`` defaults to zeros of shape
    ``(B, num_query, Hh * D)``. Cameras run one after another on the current
    stream, so the accumulation order is the reference's.
    """
    batch, num_query = count.shape
    if slots is None:
        heads, channels = value.shape[2], value.shape[3]
        slots = torch.zeros(batch, num_query, heads * channels, dtype=value.dtype, device=value.device)
    cams = value.shape[0] // batch if batch else 0
    if len(indexes) != cams:
        raise ValueError(f"got {len(indexes)} index tensors for {cams} cameras")
    for cam, index in enumerate(indexes):
        ms_deform_attn_scatter_div(value, spatial_shapes, level_start_index, sampling_locations, attention_weights,
                                   index, count, slots, cam)
    return slots


__all__ = ["ms_deform_attn_scatter_div", "sca_rebatch_scatter"]

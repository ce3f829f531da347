"""CPU oracle of SparseDrive's deformable aggregation -- TEST INFRASTRUCTURE ONLY.

A vectorised PyTorch restatement of the reference's PyTorch path
``deformable_aggregation_reference`` (``mu_space/ops/deformable_aggregation.py:113-156``):
a (pt, cam) pair contributes only when its location lies in the open square
(0, 1)^2 (the native early exit, 124-126), every scale of that camera is
sampled bilinearly at ``h = y * H - 0.5``, ``w = x * W - 0.5`` with corners
outside the map read as zero (``_bilinear_sample``, 82-110), and the sample is
multiplied channel-wise by its group weight. Gradients come from autograd, as
the reference's own CPU path gets them. Pinned by ``tests/golden/da_*.npz``,
which ``tests/golden/gen_golden_da.py`` made from the reference itself.
"""

from __future__ import annotations

import torch


def deformable_aggregation_torch(mc_ms_feat: torch.Tensor, spatial_shape: torch.Tensor,
                                 scale_start_index: torch.Tensor, sampling_location: torch.Tensor,
                                 weights: torch.Tensor) -> torch.Tensor:
    batch, _, channels = mc_ms_feat.shape
    cams, scales, _ = spatial_shape.shape
    anchors, pts = sampling_location.shape[1:3]
    groups = weights.shape[-1]
    loc_w, loc_h = sampling_location[..., 0], sampling_location[..., 1]  # (B, A, P, cams)
    inside = (loc_w > 0) & (loc_w < 1) & (loc_h > 0) & (loc_h < 1)
    out = mc_ms_feat.new_zeros(batch, anchors, channels)
    shapes = spatial_shape.tolist()
    starts = scale_start_index.tolist()
    for cam in range(cams):
        for s in range(scales):
            height, width = int(shapes[cam][s][0]), int(shapes[cam][s][1])
            start = int(starts[cam][s])
            feat = mc_ms_feat[:, start:start + height * width]  # (B, HW, C)
            h_im = loc_h[..., cam] * height - 0.5
            w_im = loc_w[..., cam] * width - 0.5
            h_low, w_low = torch.floor(h_im), torch.floor(w_im)
            lh, lw = h_im - h_low, w_im - w_low
            hh, hw = 1 - lh, 1 - lw
            sampled = 0
            for dh, dw, bil in ((0, 0, hh * hw), (0, 1, hh * lw), (1, 0, lh * hw), (1, 1, lh * lw)):
                hi, wi = h_low.long() + dh, w_low.long() + dw
                valid = (hi >= 0) & (hi <= height - 1) & (wi >= 0) & (wi <= width - 1) & inside[..., cam]
                index = (hi.clamp(0, height - 1) * width + wi.clamp(0, width - 1)).reshape(batch, -1, 1)
                corner = torch.gather(feat, 1, index.expand(-1, -1, channels)).view(batch, anchors, pts, channels)
                sampled = sampled + corner * (bil * valid)[..., None]
            channel_weights = weights[:, :, :, cam, s, :].repeat_interleave(channels // groups, dim=-1)
            out = out + (sampled * channel_weights).sum(2)
    return out


def deformable_aggregation_forward_backward(mc_ms_feat, spatial_shape, scale_start_index, sampling_location,
                                            weights, grad_output):
    """Forward output and the three gradients for ``grad_output`` (fp32, CPU)."""
    leaves = [t.detach().clone().requires_grad_(True) for t in (mc_ms_feat, sampling_location, weights)]
    out = deformable_aggregation_torch(leaves[0], spatial_shape, scale_start_index, leaves[1], leaves[2])
    out.backward(grad_output)
    return out.detach(), leaves[0].grad, leaves[1].grad, leaves[2].grad

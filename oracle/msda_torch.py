"""The reference's PyTorch MSDA formulation on CPU -- TEST INFRASTRUCTURE ONLY.

Restates ``multi_scale_deformable_attn_pytorch``
(``mu_space/ops/multi_scale_deformable_attn.py:26-58`` in the muSPACE tree): per
level, the value map of every (batch, head) is viewed as a ``(D, H_l, W_l)``
image and sampled with ``torch.nn.functional.grid_sample`` (bilinear,
``padding_mode="zeros"``, ``align_corners=False``) at ``2 * loc - 1``; the
level samples are stacked, weighted and summed over levels x points. The
arithmetic therefore lives in ATen's ``grid_sampler_2d`` (torch, third party,
pinned ``torch>=2.7,<3`` by the reference's pyproject.toml:22; this image has
2.11.0). Autograd gives the backward.

This is the CPU baseline that ``bench.py`` times (``cpu_baseline`` and the
``--impl reference`` arm) and a second, independent cross-check of the C oracle.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def msda_grid_sample(value, spatial_shapes, sampling_locations, attention_weights):
    """``(B, Lin, Hh, D)`` value -> ``(B, Lq, Hh*D)`` output, grid_sample formulation."""
    batch, _, heads, channels = value.shape
    _, queries, _, levels, points, _ = sampling_locations.shape
    sizes = [int(h) * int(w) for h, w in spatial_shapes.tolist()]
    grids = sampling_locations * 2 - 1
    per_level = []
    offset = 0
    for level, (h, w) in enumerate(spatial_shapes.tolist()):
        h, w = int(h), int(w)
        # (B, HW, Hh, D) -> (B*Hh, D, H, W)
        image = (
            value[:, offset : offset + sizes[level]]
            .permute(0, 2, 3, 1)
            .reshape(batch * heads, channels, h, w)
        )
        offset += sizes[level]
        # (B, Lq, Hh, P, 2) -> (B*Hh, Lq, P, 2)
        grid = grids[:, :, :, level].permute(0, 2, 1, 3, 4).reshape(batch * heads, queries, points, 2)
        per_level.append(
            F.grid_sample(image, grid, mode="bilinear", padding_mode="zeros", align_corners=False)
        )
    # (B*Hh, D, Lq, L, P) * (B*Hh, 1, Lq, L*P)
    stacked = torch.stack(per_level, dim=-2).flatten(-2)
    weights = attention_weights.permute(0, 2, 1, 3, 4).reshape(batch * heads, 1, queries, levels * points)
    out = (stacked * weights).sum(-1).view(batch, heads * channels, queries)
    return out.transpose(1, 2).contiguous()


def msda_grid_sample_fwd_bwd(value, spatial_shapes, sampling_locations, attention_weights, grad_output):
    """One forward + backward on CPU; returns ``(out, grad_value, grad_loc, grad_weight)``."""
    value = value.detach().requires_grad_(True)
    loc = sampling_locations.detach().requires_grad_(True)
    weight = attention_weights.detach().requires_grad_(True)
    out = msda_grid_sample(value, spatial_shapes, loc, weight)
    out.backward(grad_output)
    return out.detach(), value.grad, loc.grad, weight.grad

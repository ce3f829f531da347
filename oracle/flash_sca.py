"""CPU oracle of FlashSCA (``flash_bevpool_sca``) -- TEST INFRASTRUCTURE ONLY.

A vectorised PyTorch restatement of the reference's ``flash_bevpool_sca_reference``
(``mu_space/ops/flashbev.py:368-454``, with ``_project`` 100-113 and ``_bilinear``
116-134): for every BEV cell the voxel centre at each height is projected into
each camera (a projection counts when its depth is positive and it lands in
the image); a camera is visible when any height lands. For every channel the
output sums, over the landing (camera, height) pairs, the levels and the
points of the channel's head, ``weight * bilinear(value level map, base + offset)``
with ``base = (u / W_img * w - 0.5, v / H_img * h - 0.5)`` and zero padding, and
divides by the number of visible cameras (0 when none). Non-finite values
count as 0 (``_sanitize_value``, 56-68). Gradients (value, offsets, weights)
come from autograd. Pinned by ``tests/golden/fsca_*.npz``, made from the
reference itself by ``tests/golden/gen_golden_fsca.py``.
"""

from __future__ import annotations

import torch


def flash_sca_torch(value, projection_matrices, spatial_shapes, level_start_index, image_size, sampling_offsets,
                    attention_weights, grid_size, voxel_size, voxel_min, epsilon=1e-5):
    value = torch.where(torch.isfinite(value), value, torch.zeros_like(value))
    batch, cams, _, channels = value.shape
    gx, gy, gz = (int(v) for v in grid_size)
    heads, levels, points = sampling_offsets.shape[3], spatial_shapes.shape[0], sampling_offsets.shape[5]
    per_head = channels // heads
    image_h, image_w = (float(v) for v in image_size.tolist())
    f64 = torch.float64
    # voxel centres as the reference computes them (Python floats), then fp32
    xs = (voxel_min[0] + (torch.arange(gx, dtype=f64) + 0.5) * voxel_size[0]).float()
    ys = (voxel_min[1] + (torch.arange(gy, dtype=f64) + 0.5) * voxel_size[1]).float()
    zs = (voxel_min[2] + (torch.arange(gz, dtype=f64) + 0.5) * voxel_size[2]).float()
    X = xs.view(1, gx, 1).expand(gy, gx, gz)
    Y = ys.view(gy, 1, 1).expand(gy, gx, gz)
    Z = zs.view(1, 1, gz).expand(gy, gx, gz)
    P = projection_matrices.view(batch, cams, 3, 4)

    def row(r):  # (B, cams, gy, gx, gz)
        p = P[:, :, r]
        return (p[..., 0, None, None, None] * X + p[..., 1, None, None, None] * Y + p[..., 2, None, None, None] * Z
                + p[..., 3, None, None, None])

    depth = row(2)
    safe = torch.clamp(depth, min=epsilon)
    u, v = row(0) / safe, row(1) / safe
    lands = (depth > 0) & (u >= 0) & (u < image_w) & (v >= 0) & (v < image_h)
    visible = lands.any(-1).sum(1).to(value.dtype)  # (B, gy, gx)
    inv = torch.where(visible > 0, 1.0 / visible.clamp(min=1), torch.zeros_like(visible))

    out = value.new_zeros(batch, gy, gx, heads, per_head)
    shapes = spatial_shapes.tolist()
    starts = level_start_index.tolist()
    for cam in range(cams):
        for level in range(levels):
            h, w = int(shapes[level][0]), int(shapes[level][1])
            start = int(starts[level])
            feat = value[:, cam, start:start + h * w].view(batch, h * w, heads, per_head)
            base_u = (u[:, cam] / image_w * w - 0.5)[:, :, :, None, None, :]  # (B, gy, gx, 1, 1, gz)
            base_v = (v[:, cam] / image_h * h - 0.5)[:, :, :, None, None, :]
            su = base_u + sampling_offsets[:, :, :, :, level, :, :, 0]  # (B, gy, gx, heads, P, gz)
            sv = base_v + sampling_offsets[:, :, :, :, level, :, :, 1]
            u0, v0 = torch.floor(su), torch.floor(sv)
            du, dv = su - u0, sv - v0
            sampled = 0
            for cu, cv, bil in ((0, 0, (1 - du) * (1 - dv)), (0, 1, (1 - du) * dv), (1, 0, du * (1 - dv)),
                                (1, 1, du * dv)):
                uu, vv = u0.long() + cu, v0.long() + cv
                ok = (uu >= 0) & (uu < w) & (vv >= 0) & (vv < h)
                pix = (vv.clamp(0, h - 1) * w + uu.clamp(0, w - 1))  # (B, gy, gx, heads, P, gz)
                # gather per head: feat[b, pix, head, :]
                heads_idx = torch.arange(heads).view(1, 1, 1, heads, 1, 1).expand_as(pix)
                flat = (pix * heads + heads_idx).reshape(batch, -1, 1).expand(-1, -1, per_head)
                corner = torch.gather(feat.reshape(batch, h * w * heads, per_head), 1, flat)
                corner = corner.view(*pix.shape, per_head)
                sampled = sampled + corner * (bil * ok)[..., None]
            weight = attention_weights[:, :, :, :, level] * lands[:, cam][:, :, :, None, None, :]
            out = out + (sampled * weight[..., None]).sum(dim=(4, 5))
    return (out * inv[..., None, None]).reshape(batch, gy, gx, channels)


def flash_sca_forward_backward(value, projection_matrices, spatial_shapes, level_start_index, image_size,
                               sampling_offsets, attention_weights, grid_size, voxel_size, voxel_min, grad_output,
                               epsilon=1e-5):
    leaves = [t.detach().clone().requires_grad_(True) for t in (value, sampling_offsets, attention_weights)]
    out = flash_sca_torch(leaves[0], projection_matrices, spatial_shapes, level_start_index, image_size, leaves[1],
                          leaves[2], grid_size, voxel_size, voxel_min, epsilon)
    out.backward(grad_output)
    return out.detach(), leaves[0].grad, leaves[1].grad, leaves[2].grad

"""CPU oracle of the fused SCA scatter -- TEST INFRASTRUCTURE ONLY.

Restates ``ms_deformable_im2col_scatter_div_gpu_kernel_channels32_runtime``
(``csrc/ms_deformable_attn/ms_deform_attn_musa_kernel.muh:419-486``, launched
per camera by ``ms_deform_attn_musa.mu:455-505``): for one camera ``cam_id``,
every batch entry ``b`` and rebatched query ``q < len(index)``, the MSDA output
row of image ``b * cams + cam_id`` is multiplied by ``1 / count[b, index[q]]``
and added to ``slots[b, index[q]]``. The MSDA term comes from the C oracle
(:func:`oracle.msda_oracle.oracle_forward`, pinned to the reference's golden
vectors); the scatter arithmetic is fp32, as the kernel's ``acc_t``.
"""

from __future__ import annotations

import numpy as np

from .msda_oracle import oracle_forward


def oracle_scatter_div(value, spatial_shapes, level_start_index, sampling_locations, attention_weights, index,
                       count, slots, cam_id: int) -> np.ndarray:
    """Returns the updated copy of ``slots`` (float32) for one camera."""
    count = np.asarray(count, dtype=np.float32)
    out = np.array(slots, dtype=np.float32, copy=True)
    batch, num_query = count.shape
    cams = value.shape[0] // batch
    index = np.asarray(index, dtype=np.int64)
    valid = index.shape[0]
    if valid == 0:
        return out
    keep = (index >= 0) & (index < num_query)
    for b in range(batch):
        image = b * cams + cam_id
        rows = oracle_forward(value[image:image + 1], spatial_shapes, level_start_index,
                              np.ascontiguousarray(sampling_locations[image:image + 1, :valid]),
                              np.ascontiguousarray(attention_weights[image:image + 1, :valid]))[0]
        bev = index[keep]
        inv = np.float32(1.0) / count[b, bev]
        out[b, bev] = out[b, bev] + rows[keep] * inv[:, None]
    return out

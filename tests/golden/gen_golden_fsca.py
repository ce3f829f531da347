"""Generate the FlashSCA golden vectors from the muSPACE reference itself.

Run once, in a container that has the reference tree (it is read, never copied):

    python tests/golden/gen_golden_fsca.py <muSPACE checkout>

For every case below it builds seeded pinhole cameras around a BEV grid,
evaluates the reference's own PyTorch path
``mu_space.ops.flashbev.flash_bevpool_sca_reference`` (``mu_space/ops/flashbev.py:368-454``)
forward and, through autograd, its backward for a seeded ``grad_output``, and
stores inputs, grid parameters and outputs in ``fsca_<case>.npz``. The
reference evaluates every channel in a Python loop, so the cases are small.
"""

from __future__ import annotations

import hashlib
import importlib
import json
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _reference_fn(reference_root: str):
    sys.path.insert(0, reference_root)
    module = importlib.import_module("mu_space.ops.flashbev")
    origin = Path(module.__file__).resolve()
    if not str(origin).startswith(str(Path(reference_root).resolve())):
        raise SystemExit(f"imported {origin}, not the reference under {reference_root}")
    return module.flash_bevpool_sca_reference


def cameras(batch, cams, image_hw, gen, height=1.5):
    """Pinhole cameras at (0, 0, height) looking outwards at evenly spread yaws."""
    img_h, img_w = image_hw
    mats = torch.zeros(batch, cams, 3, 4)
    for b in range(batch):
        for c in range(cams):
            yaw = 2 * math.pi * c / cams + float(torch.randn((), generator=gen)) * 0.05
            fwd = torch.tensor([math.cos(yaw), math.sin(yaw), 0.0])
            right = torch.tensor([math.sin(yaw), -math.cos(yaw), 0.0])
            down = torch.tensor([0.0, 0.0, -1.0])
            rot = torch.stack([right, down, fwd])  # world -> camera axes
            centre = torch.tensor([0.0, 0.0, height])
            k = torch.tensor([[img_w * 0.5, 0.0, img_w * 0.5], [0.0, img_h * 0.5, img_h * 0.5], [0.0, 0.0, 1.0]])
            mats[b, c, :, :3] = k @ rot
            mats[b, c, :, 3] = k @ (-(rot @ centre))
    return mats


def _case(*, batch, cams, image_hw, shapes, stride_pad, heads, channels, points, grid, voxel_size, voxel_min, seed,
          nonfinite=False):
    gen = torch.Generator().manual_seed(seed)
    sizes = [h * w for h, w in shapes]
    stride = sum(sizes) + stride_pad
    value = torch.randn(batch, cams, stride, channels, generator=gen)
    if nonfinite:
        value[0, 0, 0, 0] = float("inf")
        value[0, 0, 1, 1] = float("nan")
        value[-1, -1, 2, 2] = float("-inf")
    proj = cameras(batch, cams, image_hw, gen)
    spatial = torch.tensor(shapes, dtype=torch.int32)
    start = torch.tensor([sum(sizes[:i]) for i in range(len(shapes))], dtype=torch.int32)
    image_size = torch.tensor(image_hw, dtype=torch.int32)
    gx, gy, gz = grid
    offsets = torch.randn(batch, gy, gx, heads, len(shapes), points, gz, 2, generator=gen) * 1.5
    weights = torch.rand(batch, gy, gx, heads, len(shapes), points, gz, generator=gen)
    return value, proj, spatial, start, image_size, offsets, weights, grid, voxel_size, voxel_min


CASES = {
    "four_cams": lambda: _case(batch=1, cams=4, image_hw=(24, 32), shapes=((6, 8), (3, 4)), stride_pad=5, heads=2,
                               channels=8, points=2, grid=(4, 4, 2), voxel_size=(2.5, 2.5, 2.0),
                               voxel_min=(-5.0, -5.0, -1.0), seed=31),
    "d32": lambda: _case(batch=1, cams=3, image_hw=(16, 24), shapes=((4, 6),), stride_pad=0, heads=2, channels=64,
                         points=2, grid=(3, 2, 2), voxel_size=(3.0, 3.0, 1.5), voxel_min=(-4.5, -3.0, -1.0), seed=32),
    "batch2_nonfinite": lambda: _case(batch=2, cams=2, image_hw=(16, 16), shapes=((4, 4), (2, 2)), stride_pad=3,
                                      heads=1, channels=4, points=3, grid=(3, 3, 3), voxel_size=(2.0, 2.0, 1.0),
                                      voxel_min=(-3.0, -3.0, -0.5), seed=33, nonfinite=True),
}


def main(reference_root: str) -> None:
    fn = _reference_fn(reference_root)
    manifest = {"generator": "tests/golden/gen_golden_fsca.py", "reference_function": "ops/flashbev.py",
                "torch": torch.__version__, "cases": {}}
    for name, make in CASES.items():
        value, proj, spatial, start, image_size, offsets, weights, grid, vsize, vmin = make()
        leaves = [value.clone().requires_grad_(True), offsets.clone().requires_grad_(True),
                  weights.clone().requires_grad_(True)]
        out = fn(leaves[0], proj, spatial, start, image_size, leaves[1], leaves[2], grid, vsize, vmin)
        grad = torch.randn(out.shape, generator=torch.Generator().manual_seed(77))
        out.backward(grad)
        arrays = {
            "value": value.numpy(), "projection_matrices": proj.numpy(), "spatial_shapes": spatial.numpy(),
            "level_start_index": start.numpy(), "image_size": image_size.numpy(),
            "sampling_offsets": offsets.numpy(), "attention_weights": weights.numpy(),
            "grid_size": np.array(grid, dtype=np.int64), "voxel_size": np.array(vsize, dtype=np.float64),
            "voxel_min": np.array(vmin, dtype=np.float64), "grad_output": grad.numpy(),
            "output": out.detach().numpy(), "grad_value": leaves[0].grad.numpy(),
            "grad_sampling_offsets": leaves[1].grad.numpy(), "grad_attention_weights": leaves[2].grad.numpy(),
        }
        path = HERE / f"fsca_{name}.npz"
        np.savez_compressed(path, **arrays)
        manifest["cases"][name] = {"sha256": hashlib.sha256(path.read_bytes()).hexdigest(),
                                   "value_shape": list(value.shape), "grid": list(grid)}
        print(name, path.stat().st_size, "bytes", "nonzero outputs", int((out != 0).sum()))
    (HERE / "FSCA_MANIFEST.json").write_text(json.dumps(manifest, indent=1) + "\n")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: gen_golden_fsca.py <muSPACE checkout>")
    main(sys.argv[1])

"""Generate the deformable-aggregation golden vectors from the muSPACE reference itself.

Run once, in a container that has the reference tree (it is read, never copied):

    python tests/golden/gen_golden_da.py <muSPACE checkout>

For every case below it draws fp32 inputs from a fixed seed, evaluates the
reference's own PyTorch path ``mu_space.ops.deformable_aggregation.deformable_aggregation_reference``
(``mu_space/ops/deformable_aggregation.py:113-156``: open-square location
test, bilinear sampling at ``y * H - 0.5`` / ``x * W - 0.5``, group weights
repeated over channels) forward and, through autograd, its backward for a
seeded ``grad_output``, and stores inputs and outputs in ``da_<case>.npz``.
``small`` is the reference test's hand-made case
(``tests/ops/test_deformable_aggregation.py:85-101``), whose second anchor sits
exactly on the excluded boundary ``x = 1``.
"""

from __future__ import annotations

import hashlib
import importlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _reference_fn(reference_root: str):
    sys.path.insert(0, reference_root)
    module = importlib.import_module("mu_space.ops.deformable_aggregation")
    origin = Path(module.__file__).resolve()
    if not str(origin).startswith(str(Path(reference_root).resolve())):
        raise SystemExit(f"imported {origin}, not the reference under {reference_root}")
    return module.deformable_aggregation_reference, str(origin)


def _small():
    mc = torch.arange(20, dtype=torch.float32).view(1, 5, 4)
    shape = torch.tensor([[[2, 2], [1, 1]]], dtype=torch.int32)
    start = torch.tensor([[0, 4]], dtype=torch.int32)
    loc = torch.tensor([[[[[0.5, 0.5]]], [[[1.0, 0.5]]]]], dtype=torch.float32)
    w = torch.tensor([[[[[[0.25, 0.5], [0.75, 1.0]]]], [[[[0.5, 0.25], [1.0, 0.75]]]]]], dtype=torch.float32)
    return mc, shape, start, loc, w


def _case(*, batch, cams, shapes, anchors, pts, channels, groups, seed, active=0.5, edges=False):
    gen = torch.Generator().manual_seed(seed)
    sizes = [h * w for h, w in shapes]
    start = torch.tensor([[sum(sizes) * c + sum(sizes[:s]) for s in range(len(shapes))] for c in range(cams)],
                         dtype=torch.int32)
    shape = torch.tensor([list(map(list, shapes))] * cams, dtype=torch.int32)
    mc = torch.randn((batch, sum(sizes) * cams, channels), generator=gen)
    pshape = (batch, anchors, pts, cams)
    inside = torch.rand(pshape + (2,), generator=gen) * 0.98 + 0.01
    outside = torch.randn(pshape + (2,), generator=gen) * 3.0
    keep = torch.rand(pshape, generator=gen) < active
    loc = torch.where(keep.unsqueeze(-1), inside, outside)
    if edges:
        # the open-square boundary and the map borders: x in {0, 1, 0.5 / W, 1 - 0.5 / W}
        h, w = shapes[0]
        xs = torch.tensor([0.0, 1.0, 0.5 / w, 1.0 - 0.5 / w, 1e-6, 1.0 - 1e-6])
        ys = torch.tensor([0.5 / h, 1.0 - 0.5 / h, 0.0, 1.0, 1.0 - 1e-6, 1e-6])
        n = min(xs.numel(), anchors * pts)
        flat = loc.view(batch, anchors * pts, cams, 2)
        flat[:, :n, 0, 0] = xs[:n]
        flat[:, :n, 0, 1] = ys[:n]
    weights = torch.rand(pshape + (len(shapes), groups), generator=gen)
    return mc, shape, start, loc, weights


CASES = {
    "small": lambda: _small(),
    "two_cams": lambda: _case(batch=2, cams=2, shapes=((6, 10), (3, 5)), anchors=7, pts=3, channels=32, groups=4,
                              seed=11),
    "sparsedrive_like": lambda: _case(batch=1, cams=6, shapes=((8, 22), (4, 11), (2, 6), (1, 3)), anchors=16,
                                      pts=13, channels=256, groups=8, seed=12, active=0.4),
    "edges": lambda: _case(batch=1, cams=2, shapes=((4, 6), (2, 3)), anchors=3, pts=2, channels=16, groups=2,
                           seed=13, edges=True),
    "odd_groups": lambda: _case(batch=2, cams=3, shapes=((5, 7),), anchors=5, pts=2, channels=24, groups=3, seed=14),
}


def main(reference_root: str) -> None:
    fn, origin = _reference_fn(reference_root)
    manifest = {"generator": "tests/golden/gen_golden_da.py", "reference_function": "ops/deformable_aggregation.py",
                "torch": torch.__version__, "cases": {}}
    for name, make in CASES.items():
        mc, shape, start, loc, w = make()
        leaves = [mc.clone().requires_grad_(True), loc.clone().requires_grad_(True), w.clone().requires_grad_(True)]
        out = fn(leaves[0], shape, start, leaves[1], leaves[2])
        grad = torch.randn(out.shape, generator=torch.Generator().manual_seed(99))
        out.backward(grad)
        arrays = {
            "mc_ms_feat": mc.numpy(), "spatial_shape": shape.numpy(), "scale_start_index": start.numpy(),
            "sampling_location": loc.numpy(), "weights": w.numpy(), "grad_output": grad.numpy(),
            "output": out.detach().numpy(), "grad_mc_ms_feat": leaves[0].grad.numpy(),
            "grad_sampling_location": leaves[1].grad.numpy(), "grad_weights": leaves[2].grad.numpy(),
        }
        path = HERE / f"da_{name}.npz"
        np.savez_compressed(path, **arrays)
        manifest["cases"][name] = {"sha256": hashlib.sha256(path.read_bytes()).hexdigest(),
                                   "mc_ms_feat_shape": list(mc.shape), "weights_shape": list(w.shape)}
        print(name, path.stat().st_size, "bytes")
    (HERE / "DA_MANIFEST.json").write_text(json.dumps(manifest, indent=1) + "\n")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: gen_golden_da.py <muSPACE checkout>")
    main(sys.argv[1])

"""FlashSCA (flash_bevpool_sca): the oracle pinned to the reference's own CPU
path, the op's validation and the C-ABI (CPU), and the sm_100a kernels against
the golden vectors and the oracle (GPU).

Mirrors the reference's ``tests/ops/test_flashbev.py`` SCA part: forward and
gradients (value, sampling offsets, attention weights) against the Python
reference, non-finite feature values read as 0, cells that no camera sees
(output 0), roi_range as an alternative to voxel_size / voxel_min, and the
validation messages.
"""

from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest
import torch

from conftest import ROOT
from muspace_b200 import cases
from muspace_b200.ops import flash_bevpool_sca
from muspace_b200.runtime import native
from oracle.flash_sca import flash_sca_forward_backward

GOLDEN = ("four_cams", "d32", "batch2_nonfinite")
TENSORS = ("value", "projection_matrices", "spatial_shapes", "level_start_index", "image_size", "sampling_offsets",
           "attention_weights")
GRADS = ("grad_value", "grad_sampling_offsets", "grad_attention_weights")


def _golden(name):
    z = np.load(ROOT / "tests" / "golden" / f"fsca_{name}.npz")
    g = {k: z[k] for k in z.files}
    t = {k: torch.from_numpy(g[k]) for k in TENSORS + ("grad_output", "output") + GRADS}
    grid = dict(grid_size=tuple(int(v) for v in g["grid_size"]), voxel_size=tuple(float(v) for v in g["voxel_size"]),
                voxel_min=tuple(float(v) for v in g["voxel_min"]))
    return t, grid


def test_golden_manifest_matches_files():
    manifest = json.loads((ROOT / "tests" / "golden" / "FSCA_MANIFEST.json").read_text())
    assert sorted(manifest["cases"]) == sorted(GOLDEN)
    for name, meta in manifest["cases"].items():
        digest = hashlib.sha256((ROOT / "tests" / "golden" / f"fsca_{name}.npz").read_bytes()).hexdigest()
        assert digest == meta["sha256"], name


@pytest.mark.parametrize("name", GOLDEN)
def test_oracle_matches_the_reference_golden_vectors(name):
    t, grid = _golden(name)
    out, *grads = flash_sca_forward_backward(*[t[k] for k in TENSORS], grid["grid_size"], grid["voxel_size"],
                                             grid["voxel_min"], t["grad_output"])
    torch.testing.assert_close(out, t["output"], rtol=1e-5, atol=1e-5)
    for got, key in zip(grads, GRADS):
        torch.testing.assert_close(got, t[key], rtol=1e-5, atol=2e-5)


def test_golden_cases_cover_unseen_cells_and_nonfinite_values():
    t, _ = _golden("batch2_nonfinite")
    assert not torch.isfinite(t["value"]).all()
    cells = t["output"].abs().sum(-1)
    assert (cells == 0).any() and (cells > 0).any()


def test_validation_mirrors_the_reference():
    t, grid = _golden("four_cams")
    args = [t[k] for k in TENSORS]
    bad = list(args)
    bad[2] = bad[2].long()
    with pytest.raises(TypeError, match="spatial_shapes must use int32"):
        flash_bevpool_sca(*bad, **grid)
    bad = list(args)
    bad[5] = bad[5][..., :1].contiguous()
    with pytest.raises(ValueError, match="invalid FlashSCA input ranks|sampling_offsets must have shape"):
        flash_bevpool_sca(*bad, **grid)
    with pytest.raises(ValueError, match="pass either roi_range or voxel_size/voxel_min"):
        flash_bevpool_sca(*args, **grid, roi_range=[0, 1, 0, 1, 0, 1])
    with pytest.raises(ValueError, match="value_stride_n must be in"):
        flash_bevpool_sca(*args, **grid, value_stride_n=10_000)
    with pytest.raises(RuntimeError, match="FlashSCA kernels need CUDA tensors"):
        flash_bevpool_sca(*args, **grid)


def test_c_abi_refuses_cpu_tensors_and_wrong_arity():
    t, grid = _golden("four_cams")
    out = torch.zeros(1, 4, 4, 8)
    fwd = native.native_function("flash_bevpool_sca_forward")
    with pytest.raises(RuntimeError, match="value must be a CUDA tensor"):
        fwd(*[t[k] for k in TENSORS], out, 2, 2, 4, 4, 2, 2.5, 2.5, 2.0, -5.0, -5.0, -1.0, t["value"].shape[2], 1e-5)
    with pytest.raises(TypeError, match="takes 19 arguments"):
        native.native_function("flash_bevpool_sca_backward")(out)


# ---------------------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------------------


@pytest.mark.gpu
@pytest.mark.parametrize("name", GOLDEN)
def test_op_matches_the_reference_golden_vectors(cuda_device, name):
    t, grid = _golden(name)
    dev = {k: t[k].to(cuda_device) for k in TENSORS}
    for k in ("value", "sampling_offsets", "attention_weights"):
        dev[k].requires_grad_(True)
    out = flash_bevpool_sca(*[dev[k] for k in TENSORS], **grid)
    out.backward(t["grad_output"].to(cuda_device))
    torch.testing.assert_close(out.detach().cpu(), t["output"], rtol=1e-4, atol=1e-4)
    for key, leaf in zip(GRADS, ("value", "sampling_offsets", "attention_weights")):
        torch.testing.assert_close(dev[leaf].grad.cpu(), t[key], rtol=1e-3, atol=1e-3)


@pytest.mark.gpu
def test_roi_range_equals_voxel_size_and_min(cuda_device):
    t, grid = _golden("four_cams")
    dev = [t[k].to(cuda_device) for k in TENSORS]
    gx, gy, gz = grid["grid_size"]
    (sx, sy, sz), (x0, y0, z0) = grid["voxel_size"], grid["voxel_min"]
    roi = [x0, x0 + gx * sx, y0, y0 + gy * sy, z0, z0 + gz * sz]
    a = flash_bevpool_sca(*dev, **grid)
    b = flash_bevpool_sca(*dev, grid["grid_size"], roi_range=roi)
    torch.testing.assert_close(a, b, rtol=1e-6, atol=1e-6)


def bevformer_inputs(device, **kw):
    return cases.flash_sca_inputs(device, **kw)


@pytest.mark.gpu
def test_bevformer_like_case_matches_the_oracle(cuda_device):
    t, kw = bevformer_inputs(cuda_device, grid=(24, 24, 4), points=4)
    leaves = list(t)
    for i in (0, 5, 6):
        leaves[i] = t[i].clone().requires_grad_(True)
    out = flash_bevpool_sca(*leaves, **kw)
    grad = torch.randn(out.shape, generator=torch.Generator().manual_seed(1)).to(cuda_device)
    out.backward(grad)
    exp = flash_sca_forward_backward(*[x.cpu() for x in t], kw["grid_size"], kw["voxel_size"], kw["voxel_min"],
                                     grad.cpu())
    assert out.abs().sum() > 0
    torch.testing.assert_close(out.detach().cpu(), exp[0], rtol=1e-4, atol=1e-4)
    for leaf, ref in zip((leaves[0], leaves[5], leaves[6]), exp[1:]):
        torch.testing.assert_close(leaf.grad.cpu(), ref, rtol=1e-3, atol=1e-3)


@pytest.mark.gpu
def test_more_landing_pairs_than_a_warp_matches_the_oracle(cuda_device):
    """6 cameras x 8 heights = 48 (camera, height) pairs per cell: the
    projection takes several rounds of the lane group, and the backward's
    level-major chunks mix pairs of several rounds."""
    t, kw = bevformer_inputs(cuda_device, grid=(12, 12, 8), points=2, seed=11)
    leaves = list(t)
    for i in (0, 5, 6):
        leaves[i] = t[i].clone().requires_grad_(True)
    out = flash_bevpool_sca(*leaves, **kw)
    grad = torch.randn(out.shape, generator=torch.Generator().manual_seed(2)).to(cuda_device)
    out.backward(grad)
    exp = flash_sca_forward_backward(*[x.cpu() for x in t], kw["grid_size"], kw["voxel_size"], kw["voxel_min"],
                                     grad.cpu())
    assert out.abs().sum() > 0
    torch.testing.assert_close(out.detach().cpu(), exp[0], rtol=1e-4, atol=1e-4)
    for leaf, ref in zip((leaves[0], leaves[5], leaves[6]), exp[1:]):
        torch.testing.assert_close(leaf.grad.cpu(), ref, rtol=1e-3, atol=1e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("grid", [(7, 5, 4), (3, 1, 4)])
def test_two_batch_entries_with_nonfinite_values_at_32_channels_a_head(cuda_device, grid):
    """32 channels a head (lane groups of 8, the BEVFormer layout) with two
    batch entries of 35 (or 3) cells each, and infinite / NaN feature values at
    pixels of the coarsest level (which every cell samples): the output and
    every gradient equal the oracle's, the non-finite values receive no
    gradient, and nothing leaks between batch entries."""
    t, kw = bevformer_inputs(cuda_device, batch=2, grid=grid, channels=64, heads=2, points=2, seed=7)
    value = t[0]
    shapes = t[2].tolist()
    start3 = int(t[3][3])
    h3, w3 = shapes[3]
    value[0, :, start3 : start3 + h3 * w3 : 7, 3] = float("inf")
    value[1, :, start3 + 3 : start3 + h3 * w3 : 11, 40] = float("nan")
    value[1, 2, 5, 33] = float("-inf")
    leaves = list(t)
    for i in (0, 5, 6):
        leaves[i] = t[i].clone().requires_grad_(True)
    out = flash_bevpool_sca(*leaves, **kw)
    grad = torch.randn(out.shape, generator=torch.Generator().manual_seed(3)).to(cuda_device)
    out.backward(grad)
    exp = flash_sca_forward_backward(*[x.cpu() for x in t], kw["grid_size"], kw["voxel_size"], kw["voxel_min"],
                                     grad.cpu())
    assert out.abs().sum() > 0 and torch.isfinite(out).all()
    torch.testing.assert_close(out.detach().cpu(), exp[0], rtol=1e-4, atol=1e-4)
    for leaf, ref in zip((leaves[0], leaves[5], leaves[6]), exp[1:]):
        assert torch.isfinite(leaf.grad).all()
        torch.testing.assert_close(leaf.grad.cpu(), ref, rtol=1e-3, atol=1e-3)
    # the non-finite values receive no gradient
    gv = leaves[0].grad
    assert (gv[0, :, start3 : start3 + h3 * w3 : 7, 3] == 0).all()
    assert (gv[1, :, start3 + 3 : start3 + h3 * w3 : 11, 40] == 0).all()

"""SparseDrive deformable aggregation: the oracle pinned to the reference's own
CPU path, the op's validation and the C-ABI (CPU), and the sm_100a kernels
against the golden vectors and the oracle (GPU).

Mirrors the reference's ``tests/ops/test_deformable_aggregation.py``: the
hand-made small case whose second anchor sits on the excluded boundary x = 1,
dtype / group validation, the feature-map format round trip, the patcher,
native vs reference at 1e-4 (forward) / 1e-3 (gradients), zero anchors, and
the production shapes (mc_ms_feat [8, 89760, 256], 6 cameras x 4 scales, 900
anchors x 13 points, 8 groups).
"""

from __future__ import annotations

import sys
import types

import numpy as np
import pytest
import torch

from conftest import ROOT
from muspace_b200 import cases
from muspace_b200.ops import deformable_aggregation, feature_maps_format
from muspace_b200.runtime import native
from oracle.deformable_aggregation import deformable_aggregation_forward_backward

GOLDEN = ("small", "two_cams", "sparsedrive_like", "edges", "odd_groups")
INPUTS = ("mc_ms_feat", "spatial_shape", "scale_start_index", "sampling_location", "weights")
GRADS = ("grad_mc_ms_feat", "grad_sampling_location", "grad_weights")


def _golden(name):
    return {k: torch.from_numpy(v) for k, v in np.load(ROOT / "tests" / "golden" / f"da_{name}.npz").items()}


def test_golden_manifest_matches_files():
    import hashlib
    import json

    manifest = json.loads((ROOT / "tests" / "golden" / "DA_MANIFEST.json").read_text())
    assert sorted(manifest["cases"]) == sorted(GOLDEN)
    for name, meta in manifest["cases"].items():
        digest = hashlib.sha256((ROOT / "tests" / "golden" / f"da_{name}.npz").read_bytes()).hexdigest()
        assert digest == meta["sha256"], name


@pytest.mark.parametrize("name", GOLDEN)
def test_oracle_matches_the_reference_golden_vectors(name):
    g = _golden(name)
    out, *grads = deformable_aggregation_forward_backward(*[g[k] for k in INPUTS], g["grad_output"])
    torch.testing.assert_close(out, g["output"], rtol=1e-5, atol=1e-5)
    for got, key in zip(grads, GRADS):
        torch.testing.assert_close(got, g[key], rtol=1e-5, atol=1e-5)


def test_small_case_ignores_the_anchor_on_the_open_boundary():
    g = _golden("small")
    assert torch.equal(g["output"][:, 1], torch.zeros_like(g["output"][:, 1]))


def _small():
    g = _golden("small")
    return [g[k].clone() for k in INPUTS]


def test_validation_mirrors_the_reference():
    t = _small()
    t[-1] = torch.ones((1, 2, 1, 1, 2, 3), dtype=torch.float32)
    with pytest.raises(ValueError, match="divisible by num_groups"):
        deformable_aggregation(*t)
    t = _small()
    t[1] = t[1].to(torch.int64)
    with pytest.raises(TypeError, match="spatial_shape must use int32"):
        deformable_aggregation(*t)
    t = _small()
    t[0] = t[0].double()
    with pytest.raises(TypeError, match="mc_ms_feat must use float32"):
        deformable_aggregation(*t)
    t = _small()
    t[-1] = torch.ones((1, 2, 1, 1, 2, 9), dtype=torch.float32)
    with pytest.raises(ValueError, match=r"num_groups must be in \[1, 8\]"):
        deformable_aggregation(*t)


def test_cpu_tensors_and_the_reference_backend_raise():
    with pytest.raises(RuntimeError, match="need CUDA tensors"):
        deformable_aggregation(*_small())
    with pytest.raises(RuntimeError, match="not part of the B200 build"):
        deformable_aggregation(*_small(), backend="reference")


def test_feature_maps_format_round_trip_preserves_values():
    levels = [
        torch.arange(1 * 2 * 4 * 2 * 3, dtype=torch.float32).view(1, 2, 4, 2, 3),
        torch.arange(1 * 2 * 4 * 1 * 2, dtype=torch.float32).view(1, 2, 4, 1, 2),
    ]
    col, shape, start = feature_maps_format(levels)
    assert col.shape == (1, 2 * (6 + 2), 4)
    assert shape.tolist() == [[[2, 3], [1, 2]]] * 2
    assert start.tolist() == [[0, 6], [8, 14]]
    # camera 1, level 1, pixel (0, 1) is row 14 + 1
    torch.testing.assert_close(col[0, 15], levels[1][0, 1, :, 0, 1])
    restored = feature_maps_format([col, shape, start], inverse=True)
    assert len(restored) == 1
    for got, expected in zip(restored[0], levels):
        torch.testing.assert_close(got, expected)


def test_c_abi_refuses_cpu_tensors_and_wrong_arity():
    t = _small()
    out = torch.zeros(1, 2, 4)
    for name in ("deformable_aggregation_forward_opt", "deformable_aggregation_forward_base"):
        with pytest.raises(RuntimeError, match="mc_ms_feat must be a CUDA tensor"):
            native.native_function(name)(*t, out)
    for name in ("deformable_aggregation_backward_opt", "deformable_aggregation_backward_base"):
        with pytest.raises(TypeError, match="takes 9 arguments"):
            native.native_function(name)(*t, out)


def test_sparsedrive_patcher_rebinds_and_restores(monkeypatch):
    from mu_space.patcher import SparseDrivePatcher

    ops = types.ModuleType("projects.mmdet3d_plugin.ops")
    blocks = types.ModuleType("projects.mmdet3d_plugin.models.blocks")

    def original(*args, **kwargs):
        return "original"

    ops.deformable_aggregation_function = original
    ops.feature_maps_format = feature_maps_format
    blocks.DAF = original
    blocks.DAF_VALID = False
    monkeypatch.setitem(sys.modules, ops.__name__, ops)
    monkeypatch.setitem(sys.modules, blocks.__name__, blocks)
    patcher = SparseDrivePatcher()
    report = patcher.apply()
    assert report.action == "applied"
    assert ops.deformable_aggregation_function is not original
    assert blocks.DAF is ops.deformable_aggregation_function
    assert blocks.DAF_VALID is True and blocks.feature_maps_format is feature_maps_format
    assert patcher.apply().action == "already-applied"
    assert patcher.restore().action == "restored"
    assert ops.deformable_aggregation_function is original and blocks.DAF is original
    assert blocks.DAF_VALID is False and not hasattr(blocks, "feature_maps_format")


def test_sparsedrive_patcher_without_the_package_is_a_patch_error(monkeypatch):
    from mu_space.patcher import PatchError, SparseDrivePatcher

    monkeypatch.setitem(sys.modules, "projects", None)
    monkeypatch.delitem(sys.modules, "projects.mmdet3d_plugin.ops", raising=False)
    with pytest.raises(PatchError, match="PYTHONPATH"):
        SparseDrivePatcher().apply()


# ---------------------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------------------


def _c_abi(t, grad, optimized):
    mc, sp, st, loc, w = t
    suffix = "opt" if optimized else "base"
    out = torch.full((mc.shape[0], loc.shape[1], mc.shape[2]), float("nan"), device=mc.device)
    native.native_function(f"deformable_aggregation_forward_{suffix}")(mc, sp, st, loc, w, out)
    gmc = torch.zeros_like(mc)
    gl = torch.full_like(loc, float("nan"))
    gw = torch.full_like(w, float("nan"))
    native.native_function(f"deformable_aggregation_backward_{suffix}")(mc, sp, st, loc, w, grad, gmc, gl, gw)
    return out, gmc, gl, gw


@pytest.mark.gpu
@pytest.mark.parametrize("optimized", [True, False])
@pytest.mark.parametrize("name", GOLDEN)
def test_kernels_match_the_reference_golden_vectors(cuda_device, name, optimized):
    g = _golden(name)
    t = [g[k].to(cuda_device) for k in INPUTS]
    got = _c_abi(t, g["grad_output"].to(cuda_device), optimized)
    torch.cuda.synchronize()
    torch.testing.assert_close(got[0].cpu(), g["output"], rtol=1e-4, atol=1e-4)
    for value, key in zip(got[1:], GRADS):
        torch.testing.assert_close(value.cpu(), g[key], rtol=1e-3, atol=1e-3)


@pytest.mark.gpu
def test_op_forward_and_backward_through_autograd(cuda_device):
    g = _golden("two_cams")
    t = [g[k].to(cuda_device) for k in INPUTS]
    for i in (0, 3, 4):
        t[i].requires_grad_(True)
    out = deformable_aggregation(*t)
    out.backward(g["grad_output"].to(cuda_device))
    torch.testing.assert_close(out.detach().cpu(), g["output"], rtol=1e-4, atol=1e-4)
    for tensor, key in zip((t[0], t[3], t[4]), GRADS):
        torch.testing.assert_close(tensor.grad.cpu(), g[key], rtol=1e-3, atol=1e-3)


@pytest.mark.gpu
def test_zero_anchors_return_empty_output_and_zero_gradients(cuda_device):
    t = [x.to(cuda_device) for x in _small()]
    t[3] = t[3][:, :0].contiguous().requires_grad_(True)
    t[4] = t[4][:, :0].contiguous().requires_grad_(True)
    t[0].requires_grad_(True)
    out = deformable_aggregation(*t)
    assert out.shape == (1, 0, 4)
    out.sum().backward()
    for tensor in (t[0], t[3], t[4]):
        assert not tensor.grad.abs().sum().item()


def _production_inputs(device, batch, anchors, seed=0):
    """The reference test's production shapes (cases.deformable_aggregation_inputs)."""
    return cases.deformable_aggregation_inputs(device, batch=batch, anchors=anchors, seed=seed)


@pytest.mark.gpu
def test_production_shapes_match_the_oracle(cuda_device):
    t, grad = _production_inputs(cuda_device, batch=2, anchors=64)
    got = _c_abi(t, grad, optimized=True)
    torch.cuda.synchronize()
    expected = deformable_aggregation_forward_backward(*[x.cpu() for x in t], grad.cpu())
    torch.testing.assert_close(got[0].cpu(), expected[0], rtol=1e-4, atol=1e-4)
    for value, ref in zip(got[1:], expected[1:]):
        torch.testing.assert_close(value.cpu(), ref, rtol=1e-3, atol=1e-3)


@pytest.mark.gpu
def test_production_shapes_opt_equals_base(cuda_device):
    """Reference test_real_shape_accuracy: the optimized pair against the
    baseline pair at the full production size (B = 8, 900 anchors)."""
    t, grad = _production_inputs(cuda_device, batch=8, anchors=900)
    opt = _c_abi(t, grad, optimized=True)
    base = _c_abi(t, grad, optimized=False)
    torch.cuda.synchronize()
    torch.testing.assert_close(opt[0], base[0], rtol=1e-4, atol=1e-4)
    for a, b in zip(opt[1:], base[1:]):
        torch.testing.assert_close(a, b, rtol=1e-3, atol=1e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("pts,cams,channels,groups", [(40, 3, 64, 4), (13, 1, 512, 8), (5, 7, 32, 2)])
def test_point_camera_and_channel_extents_match_the_oracle(cuda_device, pts, cams, channels, groups):
    """More than 32 points per camera (two compaction rounds per camera-major
    warp), a single camera, 512 channels (four lane rounds) and 7 cameras."""
    t, grad = cases.deformable_aggregation_inputs(cuda_device, batch=2, anchors=24, pts=pts, cams=cams,
                                                  channels=channels, groups=groups, active=0.6, seed=7)
    got = _c_abi(t, grad, optimized=True)
    torch.cuda.synchronize()
    expected = deformable_aggregation_forward_backward(*[x.cpu() for x in t], grad.cpu())
    torch.testing.assert_close(got[0].cpu(), expected[0], rtol=1e-4, atol=1e-4)
    for value, ref in zip(got[1:], expected[1:]):
        torch.testing.assert_close(value.cpu(), ref, rtol=1e-3, atol=1e-3)


@pytest.mark.gpu
def test_a_map_that_leaves_the_features_is_emptied_alike_in_both_kernel_pairs(cuda_device):
    """A scale whose rows would run past num_feat is emptied on the device by
    both kernel pairs, so none of its corners is read (its samples have no
    in-map corner at all): the optimized pair equals the baseline pair."""
    t, grad = cases.deformable_aggregation_inputs(cuda_device, batch=2, anchors=40, pts=13, cams=3, channels=64,
                                                  groups=4, active=0.6, seed=3)
    start = t[2].clone()
    start[1, 2] = t[0].shape[1] - 5  # the (camera 1, scale 2) map would end past the last feature row
    t[2] = start
    opt = _c_abi(t, grad, optimized=True)
    base = _c_abi(t, grad, optimized=False)
    torch.cuda.synchronize()
    assert torch.isfinite(opt[0]).all() and opt[0].abs().sum() > 0
    torch.testing.assert_close(opt[0], base[0], rtol=1e-4, atol=1e-4)
    for a, b in zip(opt[1:], base[1:]):
        torch.testing.assert_close(a, b, rtol=1e-3, atol=1e-3)


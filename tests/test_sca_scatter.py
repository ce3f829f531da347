"""Fused spatial-cross-attention scatter (MSDA forward + rebatch scatter +
camera-count normalisation), the B200 form of the reference's unexported
``ms_deformable_im2col_scatter_div_musa`` (``csrc/ms_deformable_attn/ms_deform_attn_musa.mu:455-505``,
kernel ``ms_deform_attn_musa_kernel.muh:419-486``).

CPU tests pin the oracle against an independent restatement (BEVFormer's
unfused steps on the PyTorch ``grid_sample`` formulation) and check that the
op and the C-ABI refuse bad calls before any launch. GPU tests compare the
kernel with the oracle camera by camera.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from muspace_b200.ops import ms_deform_attn_scatter_div, sca_rebatch_scatter
from muspace_b200.runtime import native
from oracle import oracle_scatter_div
from oracle.msda_torch import msda_grid_sample

FP32_TOL = 1e-4
BF16_TOL = 2e-2


def _case(seed, batch=2, cams=3, heads=2, channels=32, shapes=((6, 8), (3, 4)), points=3, max_len=9, num_query=20,
          lens=(9, 5, 0)):
    """Rebatched SCA inputs: camera c sees lens[c] distinct BEV queries."""
    rng = np.random.default_rng(seed)
    shapes = np.array(shapes, dtype=np.int64)
    start = np.concatenate([[0], np.cumsum(shapes[:, 0] * shapes[:, 1])[:-1]]).astype(np.int64)
    lin = int((shapes[:, 0] * shapes[:, 1]).sum())
    levels = len(shapes)
    f = np.float32
    indexes = [np.sort(rng.choice(num_query, size=n, replace=False)).astype(np.int64) for n in lens[:cams]]
    seen = np.zeros((num_query,), dtype=f)
    for idx in indexes:
        seen[idx] += 1
    count = np.broadcast_to(np.maximum(seen, 1.0), (batch, num_query)).astype(f).copy()
    return {
        "value": rng.standard_normal((batch * cams, lin, heads, channels)).astype(f),
        "spatial_shapes": shapes,
        "level_start_index": start,
        "sampling_locations": rng.uniform(-0.1, 1.1, (batch * cams, max_len, heads, levels, points, 2)).astype(f),
        "attention_weights": rng.uniform(0, 1, (batch * cams, max_len, heads, levels, points)).astype(f),
        "indexes": indexes,
        "count": count,
        "slots": rng.standard_normal((batch, num_query, heads * channels)).astype(f),
    }


ARGS = ("value", "spatial_shapes", "level_start_index", "sampling_locations", "attention_weights")


def _oracle_all_cameras(c):
    slots = c["slots"]
    for cam, index in enumerate(c["indexes"]):
        slots = oracle_scatter_div(*[c[k] for k in ARGS], index, c["count"], slots, cam)
    return slots


def test_oracle_matches_the_unfused_bevformer_steps():
    """BEVFormer's SCA tail on the grid_sample formulation: per camera, MSDA on
    the rebatched rows, slots[b, index] += rows; then slots /= count."""
    c = _case(seed=3)
    batch, num_query = c["count"].shape
    cams = c["value"].shape[0] // batch
    t = {k: torch.from_numpy(c[k]) for k in ARGS}
    acc = torch.zeros(batch, num_query, c["slots"].shape[2], dtype=torch.float64)
    for cam, index in enumerate(c["indexes"]):
        images = [b * cams + cam for b in range(batch)]
        rows = msda_grid_sample(t["value"][images], t["spatial_shapes"], t["sampling_locations"][images],
                                t["attention_weights"][images])
        acc[:, torch.from_numpy(index)] += rows[:, : len(index)].double()
    expected = torch.from_numpy(c["slots"]).double() + acc / torch.from_numpy(c["count"]).double()[..., None]
    got = _oracle_all_cameras(c)
    np.testing.assert_allclose(got, expected.numpy(), rtol=1e-5, atol=1e-5)


def test_oracle_skips_out_of_range_index_entries():
    c = _case(seed=4, lens=(4, 0, 0))
    index = c["indexes"][0].copy()
    index[1] = -1
    index[2] = c["count"].shape[1]
    got = oracle_scatter_div(*[c[k] for k in ARGS], index, c["count"], c["slots"], 0)
    untouched = np.ones(c["count"].shape[1], dtype=bool)
    untouched[index[[0, 3]]] = False
    np.testing.assert_array_equal(got[:, untouched], c["slots"][:, untouched])


def test_op_refuses_cpu_tensors_before_any_launch():
    c = _case(seed=5)
    t = {k: torch.from_numpy(c[k]) for k in ARGS + ("count", "slots")}
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        ms_deform_attn_scatter_div(*[t[k] for k in ARGS], torch.from_numpy(c["indexes"][0]), t["count"], t["slots"], 0)


def test_c_abi_checks_the_scatter_arguments_on_the_host():
    c = _case(seed=6)
    t = [torch.from_numpy(c[k]) for k in ARGS] + [torch.from_numpy(c["indexes"][0]),
                                                   torch.from_numpy(c["count"]), torch.from_numpy(c["slots"])]
    fn = native.native_function("ms_deform_attn_scatter_div_forward")
    with pytest.raises(RuntimeError, match="value must be a CUDA tensor"):
        fn(*t, 0)
    with pytest.raises(TypeError, match="takes 9 arguments"):
        fn(*t)


# ---------------------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------------------


def _to_device(c, device, dtype):
    out = {}
    for k in ARGS + ("count", "slots"):
        x = torch.from_numpy(c[k]).to(device)
        out[k] = x.to(dtype) if x.dtype.is_floating_point else x
    out["indexes"] = [torch.from_numpy(i).to(device) for i in c["indexes"]]
    return out


def _quantised(c, dtype):
    return {k: (torch.from_numpy(v).to(dtype).float().numpy() if isinstance(v, np.ndarray) and v.dtype == np.float32
                else v) for k, v in c.items()}


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("heads,channels", [(2, 32), (8, 32), (3, 16)])
def test_all_cameras_match_the_oracle(cuda_device, dtype, heads, channels):
    c = _quantised(_case(seed=7 + heads, heads=heads, channels=channels), dtype)
    d = _to_device(c, cuda_device, dtype)
    got = sca_rebatch_scatter(*[d[k] for k in ARGS], d["indexes"], d["count"], d["slots"])
    torch.cuda.synchronize()
    expected = _oracle_all_cameras(c)
    tol = FP32_TOL if dtype == torch.float32 else BF16_TOL
    torch.testing.assert_close(got.float().cpu(), torch.from_numpy(expected), rtol=tol, atol=tol)


@pytest.mark.gpu
def test_one_camera_leaves_other_slots_untouched(cuda_device):
    c = _case(seed=11, lens=(6, 4, 2))
    index = c["indexes"][1].copy()
    index[0] = -5  # out of range: no update
    d = _to_device(c, cuda_device, torch.float32)
    before = d["slots"].clone()
    ms_deform_attn_scatter_div(*[d[k] for k in ARGS], torch.from_numpy(index).to(cuda_device), d["count"], d["slots"], 1)
    torch.cuda.synchronize()
    expected = oracle_scatter_div(*[c[k] for k in ARGS], index, c["count"], c["slots"], 1)
    torch.testing.assert_close(d["slots"].cpu(), torch.from_numpy(expected), rtol=FP32_TOL, atol=FP32_TOL)
    touched = torch.zeros(c["count"].shape[1], dtype=torch.bool)
    touched[torch.from_numpy(index[1:])] = True
    assert torch.equal(d["slots"][:, ~touched.to(cuda_device)], before[:, ~touched.to(cuda_device)])


@pytest.mark.gpu
def test_channel_counts_without_16_byte_slices_are_refused(cuda_device):
    c = _case(seed=12, channels=5)
    d = _to_device(c, cuda_device, torch.float32)
    with pytest.raises(RuntimeError, match="16-byte lane slices"):
        ms_deform_attn_scatter_div(*[d[k] for k in ARGS], d["indexes"][0], d["count"], d["slots"], 0)

"""The staged bf16 forward (``msda_staged.cu``) on a B200.

With MUSPACE_FWD_STAGED=1 (it is opt-in: measured slower than the default
forward), bf16 calls with D = 32 and enough head-rows to give every SM four
rounds of a 1024-thread CTA (B * Hh * Lq >= SMs * 1024) take the kernel that
copies each head's smallest levels into shared memory with TMA; other calls,
and every call without the variable, take the row-wise kernel. Both add a
head-row's corners in the same order, so the staged call must equal the
row-wise one bit for bit (the whole batch, and each image run alone), and
both must match the C oracle at the bf16 tolerance of the reference's tests
(2e-2 against the fp32 oracle on identical quantised inputs).
"""

from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest
import torch

from muspace_b200 import cases
from muspace_b200.runtime import native
from oracle import oracle_forward

pytestmark = pytest.mark.gpu

INPUTS = ("value", "spatial_shapes", "level_start_index", "sampling_locations", "attention_weights")
BF16_TOL = 2e-2
HEADS = 8

# level shapes: which of them fit the 1920 staged rows (120 KB) decides what
# the kernel copies
SHAPES = {
    # BEVFormer SCA: 29x50 and 15x25 staged (1826 rows), the two larger levels from L2
    "bevformer_sca": (cases.BEVFORMER_SCA_SHAPES, 8, "clustered_oob"),
    # Deformable DETR: 25x42 and 13x21 staged
    "detr": (cases.DETR_SHAPES, 4, "uniform"),
    # levels below one 64-row box (their boxes read past the level, and past the
    # value map for the last image)
    "tiny_levels": (((60, 80), (8, 7), (3, 5), (2, 2)), 4, "uniform"),
    # one level that fits whole
    "one_level": (((40, 45),), 4, "uniform"),
    # nothing fits: the kernel runs with every level from L2
    "nothing_fits": (((100, 120), (60, 80)), 4, "uniform"),
}


def _queries(device) -> int:
    """Queries so that two images reach the staged kernel's work threshold and
    one image stays below it."""
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    need = sms * 1024
    return (need + 2 * HEADS - 1) // (2 * HEADS) + 64


def _inputs(device, name, seed=11):
    shapes, points, locations = SHAPES[name]
    cfg = cases.MSDAConfig(name, batch=2, shapes=shapes, queries=_queries(device), points=points,
                           heads=HEADS, channels=32, locations=locations)
    return cases.make_inputs(cfg, dtype=torch.bfloat16, seed=seed, device=device, with_grad=False)


def _forward(inp, staged=False):
    out = torch.empty(inp["sampling_locations"].shape[:2] + (HEADS * 32,), dtype=torch.bfloat16,
                      device=inp["value"].device)
    before = os.environ.pop("MUSPACE_FWD_STAGED", None)
    if staged:
        os.environ["MUSPACE_FWD_STAGED"] = "1"
    try:
        native.native_function("ms_deform_attn_forward")(*[inp[k] for k in INPUTS], out, 64)
    finally:
        os.environ.pop("MUSPACE_FWD_STAGED", None)
        if before is not None:
            os.environ["MUSPACE_FWD_STAGED"] = before
    return out


def _image(inp, b):
    return {k: (v if k in ("spatial_shapes", "level_start_index") else v[b : b + 1].contiguous()) for k, v in inp.items()}


def _same_bits(a, b):
    """Equal element for element, NaN where the other is NaN."""
    nan = torch.isnan(a)
    assert torch.equal(nan, torch.isnan(b))
    assert torch.equal(a[~nan], b[~nan])


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_staged_forward_equals_row_wise_and_the_oracle(cuda_device, name):
    inp = _inputs(cuda_device, name)
    out = _forward(inp, staged=True)
    _same_bits(out, _forward(inp))
    for b in (0, 1):
        _same_bits(out[b : b + 1], _forward(_image(inp, b), staged=True))
    img = _image(inp, 1)
    args = [img[k].float().cpu().numpy() if img[k].dtype.is_floating_point else img[k].cpu().numpy() for k in INPUTS]
    expected = torch.from_numpy(np.asarray(oracle_forward(*args), dtype=np.float32))
    torch.testing.assert_close(out[1:2].float().cpu(), expected, rtol=BF16_TOL, atol=BF16_TOL)


def test_staged_forward_with_non_finite_values_in_staged_and_unstaged_levels(cuda_device):
    """Inf / NaN in a staged level (BEVFormer level 3), at the first pixel of a
    staged level (the fall-back row of samples with no corner inside) and in
    an unstaged level: the exact re-sum gives the row-wise kernel's bits."""
    inp = _inputs(cuda_device, "bevformer_sca", seed=5)
    starts = cases.level_start_index(cases.BEVFORMER_SCA_SHAPES).tolist()
    value = inp["value"]
    value[0, starts[3] + 40, 2] = float("inf")
    value[1, starts[3] + 200, 5] = float("nan")
    value[:, starts[2], :] = float("-inf")
    value[1, 777, 0] = float("nan")
    out = _forward(inp, staged=True)
    assert not torch.isfinite(out.float()).all()
    _same_bits(out, _forward(inp))
    for b in (0, 1):
        _same_bits(out[b : b + 1], _forward(_image(inp, b), staged=True))


def test_staged_forward_is_deterministic_and_never_gave_up_waiting(cuda_device):
    inp = _inputs(cuda_device, "bevformer_sca", seed=3)
    first = _forward(inp, staged=True)
    for _ in range(3):
        assert torch.equal(_forward(inp, staged=True), first)
    torch.cuda.synchronize()
    lib = native.load_native_module().lib
    count = ctypes.c_uint(123)
    assert lib.msda_stage_wait_timeouts(ctypes.byref(count)) == 0
    assert count.value == 0


def test_the_variable_selects_the_staged_kernel(cuda_device):
    """The kernels a call launches (CUPTI, through the torch profiler): the
    staged one only with MUSPACE_FWD_STAGED=1, the row-wise one otherwise."""
    inp = _inputs(cuda_device, "detr", seed=9)
    launched = {}
    for staged in (False, True):
        with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA], acc_events=True) as prof:
            _forward(inp, staged=staged)
            torch.cuda.synchronize()
        launched[staged] = " ".join(e.name for e in prof.events())
    assert "forward_staged_kernel" in launched[True]
    assert "forward_vec_kernel" not in launched[True]
    assert "forward_vec_kernel" in launched[False]
    assert "forward_staged_kernel" not in launched[False]

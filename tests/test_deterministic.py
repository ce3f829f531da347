"""The deterministic MSDA backward (``ms_deform_attn_backward_deterministic``):
64-bit fixed-point sums of grad_value, bit-identical from run to run.

CPU: the work-space size and the argument checks of the C-ABI (no GPU work).
GPU: parity with the C oracle on every lane layout the row-wise kernels take
(and the scalar kernel), bit-identical grad_value across repeated calls at a
BEVFormer-base size where the default backward's REDs land in varying order,
agreement with the default backward, the autograd path under
``torch.use_deterministic_algorithms(True)``, and non-finite grad_output.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from muspace_b200 import cases
from muspace_b200.runtime import native
from oracle import oracle_backward

INPUTS = ("value", "spatial_shapes", "level_start_index", "sampling_locations", "attention_weights")


def test_workspace_is_header_plus_one_int64_per_grad_value_element():
    assert native.deterministic_workspace_bytes(48, 30825, 8, 32, 4, 10000, 8) == 256 + 8 * 48 * 30825 * 8 * 32
    assert native.deterministic_workspace_bytes(0, 0, 0, 0, 0, 0, 0) == 256
    with pytest.raises(RuntimeError, match="non-negative"):
        native.deterministic_workspace_bytes(-1, 1, 1, 1, 1, 1, 1)


def test_plain_pointer_entry_rejects_a_short_or_misaligned_workspace():
    """Both checks fail on the host, before any CUDA call (the pointers are
    never dereferenced)."""
    lib = native.load_native_module().lib
    fn = lib.msda_backward_deterministic
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int, ctypes.POINTER(native.MsdaDims)] + [ctypes.c_void_p] * 10 + [ctypes.c_size_t,
                                                                                                  ctypes.c_void_p]
    dims = native.MsdaDims(1, 4, 1, 4, 1, 2, 1)
    fake = [ctypes.c_void_p(4096)] * 9
    need = native.deterministic_workspace_bytes(1, 4, 1, 4, 1, 2, 1)
    assert fn(0, ctypes.byref(dims), *fake, ctypes.c_void_p(4096), need - 1, None) != 0
    assert "workspace holds" in lib.msda_last_error().decode()
    assert fn(0, ctypes.byref(dims), *fake, ctypes.c_void_p(4096 + 8), need, None) != 0
    assert "256-byte aligned" in lib.msda_last_error().decode()


def test_dlpack_entry_refuses_cpu_tensors():
    fn = native.native_function("ms_deform_attn_backward_deterministic")
    t = [torch.zeros(1, 4, 1, 4), torch.tensor([[2, 2]]), torch.tensor([0]), torch.zeros(1, 2, 1, 1, 1, 2),
         torch.zeros(1, 2, 1, 1, 1), torch.zeros(1, 2, 4), torch.zeros(1, 4, 1, 4), torch.zeros(1, 2, 1, 1, 1, 2),
         torch.zeros(1, 2, 1, 1, 1), torch.zeros(512, dtype=torch.uint8)]
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        fn(*t, 64)


# ---------------------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------------------


def _deterministic(inp, grad_output):
    t = [inp[k] for k in INPUTS]
    dev = t[0].device
    gv = torch.zeros(t[0].shape, dtype=torch.float32, device=dev)
    gl = torch.full(t[3].shape, float("nan"), dtype=torch.float32, device=dev)
    gw = torch.full(t[4].shape, float("nan"), dtype=torch.float32, device=dev)
    b, lin, hh, d = t[0].shape
    _, lq, _, levels, points, _ = t[3].shape
    ws = torch.empty(native.deterministic_workspace_bytes(b, lin, hh, d, levels, lq, points), dtype=torch.uint8,
                     device=dev)
    native.native_function("ms_deform_attn_backward_deterministic")(*t, grad_output.contiguous(), gv, gl, gw, ws, 64)
    return gv, gl, gw


def _default(inp, grad_output):
    t = [inp[k] for k in INPUTS]
    dev = t[0].device
    gv = torch.zeros(t[0].shape, dtype=torch.float32, device=dev)
    gl = torch.empty(t[3].shape, dtype=torch.float32, device=dev)
    gw = torch.empty(t[4].shape, dtype=torch.float32, device=dev)
    native.native_function("ms_deform_attn_backward")(*t, grad_output.contiguous(), gv, gl, gw, 64)
    return gv, gl, gw


def _random_case(channels, levels, points, seed, batch=2, queries=9, heads=2):
    rng = np.random.default_rng(seed)
    shapes = np.array([(5, 7), (3, 4), (2, 2), (1, 3)][:levels], dtype=np.int64)
    start = np.concatenate([[0], np.cumsum(shapes[:, 0] * shapes[:, 1])[:-1]]).astype(np.int64)
    lin = int((shapes[:, 0] * shapes[:, 1]).sum())
    f = np.float32
    return {
        "value": rng.standard_normal((batch, lin, heads, channels)).astype(f),
        "spatial_shapes": shapes,
        "level_start_index": start,
        "sampling_locations": rng.uniform(-0.1, 1.1, (batch, queries, heads, levels, points, 2)).astype(f),
        "attention_weights": rng.uniform(0, 1, (batch, queries, heads, levels, points)).astype(f),
        "grad_output": rng.standard_normal((batch, queries, heads * channels)).astype(f),
    }


@pytest.mark.gpu
@pytest.mark.parametrize("channels", [5, 16, 32, 64])
@pytest.mark.parametrize("levels,points", [(1, 4), (4, 2), (3, 3)])
def test_matches_the_c_oracle(cuda_device, channels, levels, points):
    """D = 5 takes the scalar kernel for grad_loc / grad_w, the others the
    vector and lane-pair kernels (bf16 D = 16 / 32 with more than 4 samples)."""
    g = _random_case(channels, levels, points, seed=channels * 7 + levels * 3 + points)
    for dtype in (torch.float32, torch.bfloat16):
        q = {k: (torch.from_numpy(v).to(dtype).float().numpy() if v.dtype == np.float32 else v) for k, v in g.items()}
        exp_gv, exp_gl, exp_gw = oracle_backward(*[q[k] for k in INPUTS], q["grad_output"])
        inp = {k: torch.from_numpy(v).to(cuda_device) for k, v in q.items()}
        inp = {k: (v.to(dtype) if v.dtype.is_floating_point else v) for k, v in inp.items()}
        gv, gl, gw = _deterministic(inp, inp["grad_output"])
        torch.cuda.synchronize()
        for got, exp, what in ((gv, exp_gv, "grad_value"), (gl, exp_gl, "grad_loc"), (gw, exp_gw, "grad_w")):
            torch.testing.assert_close(got.cpu(), torch.from_numpy(exp), rtol=1e-4, atol=1e-4,
                                       msg=lambda m: f"D={channels} L={levels} P={points} {dtype} {what}: {m}")


@pytest.mark.gpu
def test_grad_value_is_bit_identical_across_calls(cuda_device):
    """c2 shapes (6 camera images, bf16): clustered samples put hundreds of
    contributions on the coarse levels' pixels. The deterministic path repeats
    bit for bit and agrees with the default path to fp32 accumulation error."""
    cfg = cases.CONFIGS["c2"]
    inp = cases.make_inputs(cfg, dtype=torch.bfloat16, device=cuda_device)
    first = _deterministic(inp, inp["grad_output"])
    for _ in range(3):
        again = _deterministic(inp, inp["grad_output"])
        for a, b in zip(first, again):
            assert torch.equal(a, b)
    default = _default(inp, inp["grad_output"])
    torch.cuda.synchronize()
    scale = first[0].abs().max()
    assert (first[0] - default[0]).abs().max() <= 1e-5 * scale
    assert torch.equal(first[1], default[1]) and torch.equal(first[2], default[2])


@pytest.mark.gpu
def test_autograd_uses_it_under_deterministic_algorithms(cuda_device):
    from mu_space import multi_scale_deformable_attn

    g = _random_case(32, 4, 4, seed=3, queries=64, heads=4)
    inp = {k: torch.from_numpy(v).to(cuda_device) for k, v in g.items()}
    grads = []
    for deterministic in (True, True, False):
        leaves = [inp[k].clone().requires_grad_(inp[k].dtype.is_floating_point) for k in INPUTS]
        torch.use_deterministic_algorithms(deterministic)
        try:
            out = multi_scale_deformable_attn(*leaves)
            out.backward(inp["grad_output"])
        finally:
            torch.use_deterministic_algorithms(False)
        grads.append([leaves[i].grad for i in (0, 3, 4)])
    for a, b in zip(grads[0], grads[1]):
        assert torch.equal(a, b)
    for a, b in zip(grads[0], grads[2]):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5)


@pytest.mark.gpu
def test_non_finite_grad_output_gives_the_default_paths_non_finite_elements(cuda_device):
    g = _random_case(32, 2, 4, seed=9, queries=16)
    inp = {k: torch.from_numpy(v).to(cuda_device) for k, v in g.items()}
    grad = inp["grad_output"].clone()
    grad[0, 3, 5] = float("inf")
    grad[1, 7, 40] = float("nan")
    det = _deterministic(inp, grad)
    ref = _default(inp, grad)
    torch.cuda.synchronize()
    assert not torch.isfinite(det[0]).all()
    assert torch.equal(torch.isfinite(det[0]), torch.isfinite(ref[0]))
    finite = torch.isfinite(ref[0])
    torch.testing.assert_close(det[0][finite], ref[0][finite], rtol=1e-5, atol=1e-5)

"""Parity of the sm_100a MSDA kernels with the reference, on a B200.

Small cases compare against the golden vectors made by the reference's own
PyTorch path and against the C oracle; BASELINE-sized cases compare a random
subset of head-rows against the C oracle and check size-independent
properties (batch slicing, query additivity of grad_value, determinism).

Tolerances are the reference's own (``tests/ops/test_multi_scale_deformable_attn.py``):
max-abs/rel 1e-4 for fp32 storage, 2e-2 against the fp32 oracle for bf16
storage on identical bf16-quantised inputs, 1e-2 for float16 (computed in fp32).
"""

from __future__ import annotations

from importlib import import_module

import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from mu_space import clear_dispatch_report, get_last_dispatch_report, multi_scale_deformable_attn
from muspace_b200 import cases
from muspace_b200.runtime import native
from oracle import oracle_backward, oracle_forward

pytestmark = pytest.mark.gpu
msda_module = import_module("mu_space.ops.multi_scale_deformable_attn")

FP32_TOL = 1e-4
BF16_TOL = 2e-2
INPUTS = ("value", "spatial_shapes", "level_start_index", "sampling_locations", "attention_weights")


def _to(g, device, dtype=torch.float32, grad=True):
    out = []
    for key in INPUTS:
        t = torch.from_numpy(g[key]).to(device)
        if t.dtype.is_floating_point:
            t = t.to(dtype)
            if grad:
                t.requires_grad_(True)
        out.append(t)
    return out


def _fwd_bwd(tensors, grad_output, backend="cuda"):
    out = multi_scale_deformable_attn(*tensors, backend=backend)
    out.backward(grad_output.to(out.dtype))
    return out, tensors[0].grad, tensors[3].grad, tensors[4].grad


def _close(actual, expected, tol, what):
    a = actual.detach().float().cpu()
    e = torch.as_tensor(expected).float()
    torch.testing.assert_close(a, e, rtol=tol, atol=tol, msg=lambda m: f"{what}: {m}")


@pytest.mark.parametrize("name", [n for n in golden_names() if not n.endswith("bf16q")])
def test_fp32_forward_backward_matches_reference_golden(cuda_device, name):
    g = load_golden(name)
    tensors = _to(g, cuda_device)
    grad = torch.from_numpy(g["grad_output"]).to(cuda_device)
    out, gv, gl, gw = _fwd_bwd(tensors, grad)
    _close(out, g["output"], FP32_TOL, f"{name}:output")
    _close(gv, g["grad_value"], FP32_TOL, f"{name}:grad_value")
    _close(gl, g["grad_sampling_locations"], FP32_TOL, f"{name}:grad_loc")
    _close(gw, g["grad_attention_weights"], FP32_TOL, f"{name}:grad_w")


@pytest.mark.parametrize("name", ["c0_small_bf16q", "c2_small_bf16q", "c0_small", "c2_small", "c4_small_oob", "edges"])
def test_bf16_storage_matches_fp32_reference(cuda_device, name):
    """Reference test 378-424: bf16 storage costs no more than bf16 rounding of
    the results; the oracle evaluates the same quantised inputs in fp32."""
    g = load_golden(name)
    quantised = {k: (v if v.dtype != np.float32 else torch.from_numpy(v).to(torch.bfloat16).float().numpy()) for k, v in g.items()}
    args = [quantised[k] for k in INPUTS]
    exp_out = oracle_forward(*args)
    exp_gv, exp_gl, exp_gw = oracle_backward(*args, quantised["grad_output"])
    tensors = _to(quantised, cuda_device, torch.bfloat16)
    grad = torch.from_numpy(quantised["grad_output"]).to(cuda_device, torch.bfloat16)
    clear_dispatch_report()
    out, gv, gl, gw = _fwd_bwd(tensors, grad)
    assert out.dtype == torch.bfloat16
    assert get_last_dispatch_report().selected_backend == "cuda"
    _close(out, exp_out, BF16_TOL, f"{name}:output")
    _close(gv, exp_gv, BF16_TOL, f"{name}:grad_value")
    _close(gl, exp_gl, BF16_TOL, f"{name}:grad_loc")
    _close(gw, exp_gw, BF16_TOL, f"{name}:grad_w")


@pytest.mark.parametrize("name", ["c1_small", "c3_small", "ragged_d16", "odd_d5", "wide_d64", "edges", "ref_fixture_c"])
def test_c_abi_matches_c_oracle(cuda_device, name):
    """Straight through the DLPack C-ABI (no autograd), both dtypes."""
    g = load_golden(name)
    for dtype, tol in ((torch.float32, FP32_TOL), (torch.bfloat16, BF16_TOL)):
        q = {k: (torch.from_numpy(v).to(dtype).float().numpy() if v.dtype == np.float32 else v) for k, v in g.items()}
        args = [q[k] for k in INPUTS]
        exp_out = oracle_forward(*args)
        exp_gv, exp_gl, exp_gw = oracle_backward(*args, q["grad_output"])
        t = [torch.from_numpy(q[k]).to(cuda_device) for k in INPUTS]
        t = [x.to(dtype) if x.dtype.is_floating_point else x for x in t]
        grad = torch.from_numpy(q["grad_output"]).to(cuda_device, dtype)
        out = torch.empty(grad.shape, dtype=dtype, device=cuda_device)
        native.native_function("ms_deform_attn_forward")(*t, out, 64)
        gv = torch.zeros(t[0].shape, dtype=torch.float32, device=cuda_device)
        gl = torch.full(t[3].shape, float("nan"), dtype=torch.float32, device=cuda_device)
        gw = torch.full(t[4].shape, float("nan"), dtype=torch.float32, device=cuda_device)
        native.native_function("ms_deform_attn_backward")(*t, grad, gv, gl, gw, 64)
        torch.cuda.synchronize()
        _close(out, exp_out, tol, f"{name}/{dtype}:output")
        # the gradient buffers are fp32 whatever the storage dtype: fp32 tolerance
        _close(gv, exp_gv, FP32_TOL, f"{name}/{dtype}:grad_value")
        # grad_loc / grad_w are overwritten everywhere (no NaN left from the fill)
        _close(gl, exp_gl, FP32_TOL, f"{name}/{dtype}:grad_loc")
        _close(gw, exp_gw, FP32_TOL, f"{name}/{dtype}:grad_w")


def _random_case(channels, levels, points, seed, batch=2, queries=7, heads=2):
    """Seeded inputs with locations spread over [-0.1, 1.1] (some corners and
    samples outside their level)."""
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


@pytest.mark.parametrize("channels", [4, 8, 16, 32, 128, 256])
@pytest.mark.parametrize("levels,points", [(3, 3), (1, 1), (4, 2), (2, 7), (4, 13)])
def test_every_lane_layout_matches_c_oracle(cuda_device, channels, levels, points):
    """Head-rows of 4..256 channels take every lane layout of the vector
    kernels (1 to 32 lanes of 8 or 16 bytes, the lane-pair backward for bf16
    D = 16 / 32 with more than 4 samples, and the scalar kernels for fp32
    D = 256); 1, 8, 9, 14 and 52 samples per head-row cover a chunk of staged
    samples that is partly empty, exactly full, or followed by a short one, and
    point counts that are not powers of two (the level of a sample comes from
    a multiply-high by a host constant, not a division)."""
    g = _random_case(channels, levels, points, seed=channels * 100 + levels * 10 + points)
    for dtype, tol in ((torch.float32, FP32_TOL), (torch.bfloat16, BF16_TOL)):
        q = {k: (torch.from_numpy(v).to(dtype).float().numpy() if v.dtype == np.float32 else v) for k, v in g.items()}
        args = [q[k] for k in INPUTS]
        exp_out = oracle_forward(*args)
        exp_gv, exp_gl, exp_gw = oracle_backward(*args, q["grad_output"])
        inp = {k: torch.from_numpy(v).to(cuda_device) for k, v in q.items()}
        inp = {k: (v.to(dtype) if v.dtype.is_floating_point else v) for k, v in inp.items()}
        out, (gv, gl, gw) = _c_abi_fwd_bwd(inp, dtype)
        torch.cuda.synchronize()
        what = f"D={channels} L={levels} P={points} {dtype}"
        _close(out, exp_out, tol, f"{what}:output")
        _close(gv, exp_gv, FP32_TOL, f"{what}:grad_value")
        _close(gl, exp_gl, FP32_TOL, f"{what}:grad_loc")
        _close(gw, exp_gw, FP32_TOL, f"{what}:grad_w")


def test_bf16_keeps_sampling_geometry_in_fp32(cuda_device):
    """Reference test 430-468: pixels 499 | 500 hold 0 | 4096, x = 499.5 -> 2048."""
    width = 1000
    value = torch.zeros(1, width, 1, 1, dtype=torch.bfloat16, device=cuda_device)
    value[:, width // 2 :] = 4096.0
    shapes = torch.tensor([[1, width]], dtype=torch.int64, device=cuda_device)
    start = torch.zeros(1, dtype=torch.int64, device=cuda_device)
    loc = torch.full((1, 1, 1, 1, 1, 2), 0.5, dtype=torch.bfloat16, device=cuda_device)
    weights = torch.ones(1, 1, 1, 1, 1, dtype=torch.bfloat16, device=cuda_device)
    out = multi_scale_deformable_attn(value, shapes, start, loc, weights)
    assert out.float().item() == 2048.0


def test_out_of_range_samples_are_zero_with_zero_gradients(cuda_device):
    g = load_golden("all_oob")
    tensors = _to(g, cuda_device)
    out, gv, gl, gw = _fwd_bwd(tensors, torch.ones(1, 2, 2, device=cuda_device))
    for t in (out, gv, gl, gw):
        assert not t.detach().abs().sum().item()


def test_zero_queries_returns_empty_output_and_zero_gradients(cuda_device):
    g = load_golden("ref_fixture_a")
    tensors = _to(g, cuda_device)
    tensors[3] = tensors[3].detach()[:, :0].requires_grad_(True)
    tensors[4] = tensors[4].detach()[:, :0].requires_grad_(True)
    out = multi_scale_deformable_attn(*tensors)
    assert out.shape == (1, 0, 6)
    out.sum().backward()
    for i in (0, 3, 4):
        assert tensors[i].grad is not None and not tensors[i].grad.abs().sum().item()


class _NativeCallSpy:
    def __init__(self, inner):
        self._inner = inner
        self.calls = []

    def __getattr__(self, name):
        target = getattr(self._inner, name)

        def recorded(*args):
            self.calls.append((name, [getattr(a, "dtype", None) for a in args]))
            return target(*args)

        return recorded


def test_bf16_reaches_the_kernel_as_bfloat16(cuda_device, monkeypatch):
    """Reference test 333-372: storage dtype at the FFI, fp32 accumulators."""
    spy = _NativeCallSpy(msda_module._native_extension())
    monkeypatch.setattr(msda_module, "_native_extension", lambda: spy)
    g = load_golden("ref_fixture_b")
    tensors = _to(g, cuda_device, torch.bfloat16)
    multi_scale_deformable_attn(*tensors).float().sum().backward()
    assert [n for n, _ in spy.calls] == ["ms_deform_attn_forward", "ms_deform_attn_backward"]
    assert spy.calls[0][1][:6] == [torch.bfloat16, torch.int64, torch.int64, torch.bfloat16, torch.bfloat16, torch.bfloat16]
    assert spy.calls[1][1][5:9] == [torch.bfloat16, torch.float32, torch.float32, torch.float32]


def test_float16_is_computed_in_fp32(cuda_device):
    g = load_golden("ref_fixture_c")
    tensors = _to(g, cuda_device, torch.float16)
    out = multi_scale_deformable_attn(*tensors)
    assert out.dtype == torch.float16
    _close(out, g["output"], 1e-2, "fp16 output")


def test_noncontiguous_inputs(cuda_device):
    g = load_golden("c1_small")
    value = torch.zeros(*g["value"].shape, 2, device=cuda_device)
    value[..., 0] = torch.from_numpy(g["value"]).to(cuda_device)
    loc = torch.zeros(*g["sampling_locations"].shape, 2, device=cuda_device)
    loc[..., 0] = torch.from_numpy(g["sampling_locations"]).to(cuda_device)
    value, loc = value[..., 0], loc[..., 0]
    assert not value.is_contiguous() and not loc.is_contiguous()
    shapes = torch.from_numpy(g["spatial_shapes"]).to(cuda_device)
    start = torch.from_numpy(g["level_start_index"]).to(cuda_device)
    weights = torch.from_numpy(g["attention_weights"]).to(cuda_device)
    out = multi_scale_deformable_attn(value, shapes, start, loc, weights)
    _close(out, g["output"], FP32_TOL, "noncontiguous output")


def test_host_side_shape_tables_are_moved_to_the_device(cuda_device):
    g = load_golden("c1_small")
    tensors = _to(g, cuda_device, grad=False)
    tensors[1], tensors[2] = tensors[1].cpu(), tensors[2].cpu()
    out = multi_scale_deformable_attn(*tensors)
    _close(out, g["output"], FP32_TOL, "cpu shape tables")


def test_im2col_step_rules(cuda_device):
    g = load_golden("c1_small")  # batch 2
    tensors = _to(g, cuda_device, grad=False)
    ref = multi_scale_deformable_attn(*tensors, im2col_step=64)
    for step in (1, 2, 3):
        torch.testing.assert_close(multi_scale_deformable_attn(*tensors, im2col_step=step), ref, rtol=0, atol=0)
    three = [torch.cat([t, t[:1]]) if i in (0, 3, 4) else t for i, t in enumerate(tensors)]
    with pytest.raises(RuntimeError, match="divisible by im2col_step"):
        multi_scale_deformable_attn(*three, im2col_step=2)


def test_native_library_is_the_code_that_ran(cuda_device):
    g = load_golden("ref_fixture_a")
    multi_scale_deformable_attn(*_to(g, cuda_device, grad=False))
    torch.cuda.synchronize()
    maps = open("/proc/self/maps").read()
    assert "libmuspace_ops.so" in maps


# ---------------------------------------------------------------------------------------
# BASELINE-sized cases
# ---------------------------------------------------------------------------------------


def _subset_check(inputs, out, grads, dtype_tol, rows=48, seed=0):
    """Compare `rows` random (b, q) query rows (all heads) against the C oracle."""
    b, lq = inputs["sampling_locations"].shape[:2]
    rng = np.random.default_rng(seed)
    picks = [(int(rng.integers(b)), int(rng.integers(lq))) for _ in range(rows)]
    value = inputs["value"].float().cpu().numpy()
    shapes = inputs["spatial_shapes"].cpu().numpy()
    start = inputs["level_start_index"].cpu().numpy()
    for bi, qi in picks:
        loc = inputs["sampling_locations"][bi : bi + 1, qi : qi + 1].float().cpu().numpy()
        w = inputs["attention_weights"][bi : bi + 1, qi : qi + 1].float().cpu().numpy()
        g = inputs["grad_output"][bi : bi + 1, qi : qi + 1].float().cpu().numpy()
        exp = oracle_forward(value[bi : bi + 1], shapes, start, loc, w)
        _, exp_gl, exp_gw = oracle_backward(value[bi : bi + 1], shapes, start, loc, w, g)
        _close(out[bi : bi + 1, qi : qi + 1], exp, dtype_tol, f"row {bi},{qi} output")
        # fp32 gradient buffers from identical (quantised) inputs: fp32 tolerance
        _close(grads[1][bi : bi + 1, qi : qi + 1], exp_gl, FP32_TOL, f"row {bi},{qi} grad_loc")
        _close(grads[2][bi : bi + 1, qi : qi + 1], exp_gw, FP32_TOL, f"row {bi},{qi} grad_w")


def _c_abi_fwd_bwd(inp, dtype):
    t = [inp[k] for k in INPUTS]
    out = torch.empty(inp["grad_output"].shape, dtype=dtype, device=t[0].device)
    native.native_function("ms_deform_attn_forward")(*t, out, 64)
    gv = torch.zeros(t[0].shape, dtype=torch.float32, device=t[0].device)
    gl = torch.empty(t[3].shape, dtype=torch.float32, device=t[0].device)
    gw = torch.empty(t[4].shape, dtype=torch.float32, device=t[0].device)
    native.native_function("ms_deform_attn_backward")(*t, inp["grad_output"].contiguous(), gv, gl, gw, 64)
    return out, (gv, gl, gw)


@pytest.mark.parametrize(
    "config,dtype",
    [("c1", torch.float32), ("c1", torch.bfloat16), ("c2", torch.bfloat16), ("c3", torch.bfloat16),
     ("bevformer-1l", torch.float32), ("bevformer-1l", torch.bfloat16)],
)
def test_baseline_sizes_match_oracle_on_sampled_rows(cuda_device, config, dtype):
    cfg = cases.CONFIGS[config]
    inp = cases.make_inputs(cfg, dtype=dtype, device=cuda_device)
    out, grads = _c_abi_fwd_bwd(inp, dtype)
    torch.cuda.synchronize()
    tol = FP32_TOL if dtype == torch.float32 else BF16_TOL
    _subset_check(inp, out, grads, tol)
    # forward is deterministic
    out2, _ = _c_abi_fwd_bwd(inp, dtype)
    assert torch.equal(out, out2)


def _image_check(inp, out, grads, b, dtype_tol, what):
    """Every element of image b -- output, grad_value, grad_loc, grad_w --
    against the C oracle run on that image alone (an image's head-rows only
    read its own value map and only write its own grad_value)."""
    img = {k: (v if k in ("spatial_shapes", "level_start_index") else v[b : b + 1]) for k, v in inp.items()}
    args = [img[k].float().cpu().numpy() if img[k].dtype.is_floating_point else img[k].cpu().numpy() for k in INPUTS]
    exp_out = oracle_forward(*args)
    exp_gv, exp_gl, exp_gw = oracle_backward(*args, img["grad_output"].float().cpu().numpy())
    gv, gl, gw = (g[b : b + 1] for g in grads)
    _close(out[b : b + 1], exp_out, dtype_tol, f"{what} image {b} output")
    # fp32 gradient buffers from identical (quantised) inputs: fp32 tolerance
    _close(gv, exp_gv, FP32_TOL, f"{what} image {b} grad_value")
    _close(gl, exp_gl, FP32_TOL, f"{what} image {b} grad_loc")
    _close(gw, exp_gw, FP32_TOL, f"{what} image {b} grad_w")


@pytest.mark.parametrize(
    "config,dtype,images",
    [("c2", torch.bfloat16, (0, 5)), ("c4", torch.bfloat16, (0, 23)), ("c1", torch.float32, (1,)),
     ("c1", torch.bfloat16, (0,)), ("c3", torch.bfloat16, (1,)), ("bevformer-1l", torch.float32, (0,))],
)
def test_baseline_sizes_match_oracle_on_whole_images(cuda_device, config, dtype, images):
    """The full batched launch at the BASELINE size, then every element of
    whole camera images (all queries, all heads) against the C oracle,
    grad_value included: dense images are where many samples of different
    queries land on one pixel row and the backward's folded / merged
    reductions meet."""
    cfg = cases.CONFIGS[config]
    inp = cases.make_inputs(cfg, dtype=dtype, device=cuda_device)
    out, grads = _c_abi_fwd_bwd(inp, dtype)
    torch.cuda.synchronize()
    tol = FP32_TOL if dtype == torch.float32 else BF16_TOL
    for b in images:
        _image_check(inp, out, grads, b, tol, config)


def test_c0_full_size_matches_oracle_everywhere(cuda_device):
    """Config 0 at its stated size (Lin = Lq = 1360, fp32): every output and
    gradient element, through the public autograd op and through the C-ABI."""
    cfg = cases.CONFIGS["c0"]
    inp = cases.make_inputs(cfg, dtype=torch.float32, device=cuda_device)
    out, grads = _c_abi_fwd_bwd(inp, torch.float32)
    torch.cuda.synchronize()
    _image_check(inp, out, grads, 0, FP32_TOL, "c0")
    tensors = [inp[k].clone().requires_grad_(inp[k].dtype.is_floating_point) for k in INPUTS]
    o, gv, gl, gw = _fwd_bwd(tensors, inp["grad_output"])
    torch.testing.assert_close(o, out, rtol=0, atol=0)
    for got, want, name in ((gv, grads[0], "grad_value"), (gl, grads[1], "grad_loc"), (gw, grads[2], "grad_w")):
        torch.testing.assert_close(got, want, rtol=FP32_TOL, atol=FP32_TOL, msg=lambda m, name=name: f"c0 {name}: {m}")


def test_c4_batch_slices_equal_the_whole_and_grad_value_is_additive(cuda_device):
    """Size-independent properties at the full c4 size (B=48, bf16): per-camera
    slices reproduce the batched call exactly (forward, grad_loc, grad_w) and
    grad_value of the two query halves adds up to the whole."""
    cfg = cases.CONFIGS["c4"]
    inp = cases.make_inputs(cfg, dtype=torch.bfloat16, device=cuda_device)
    out, (gv, gl, gw) = _c_abi_fwd_bwd(inp, torch.bfloat16)
    for b in (0, 17, 47):
        part = {k: (v[b : b + 1] if k not in ("spatial_shapes", "level_start_index") else v) for k, v in inp.items()}
        o, (pgv, pgl, pgw) = _c_abi_fwd_bwd(part, torch.bfloat16)
        assert torch.equal(o, out[b : b + 1])
        assert torch.equal(pgl, gl[b : b + 1])
        assert torch.equal(pgw, gw[b : b + 1])
        torch.testing.assert_close(pgv, gv[b : b + 1], rtol=1e-5, atol=1e-5)
    half = cfg.queries // 2
    total = torch.zeros_like(gv)
    for sl in (slice(0, half), slice(half, None)):
        part = dict(inp)
        for k in ("sampling_locations", "attention_weights", "grad_output"):
            part[k] = inp[k][:, sl].contiguous()
        _, (pgv, _, _) = _c_abi_fwd_bwd(part, torch.bfloat16)
        total += pgv
    torch.testing.assert_close(total, gv, rtol=1e-4, atol=1e-4)
    _subset_check(inp, out, (gv, gl, gw), BF16_TOL, rows=24, seed=1)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_non_finite_values_next_to_out_of_level_corners(cuda_device, dtype):
    """Infinite and NaN values at pixel 0 and along a border, with samples
    half outside their level: the forward (whose bf16 kernels gather an
    out-of-level corner from an in-level row with weight 0, and sum a head-row
    again the exact way when its sum is not finite) matches the oracle
    element for element, non-finite elements included."""
    g = _random_case(32, 3, 3, seed=77, queries=40, heads=2)
    value = g["value"].copy()
    value[:, 0] = np.inf            # row 0 of level 0 (the fall-back row of fully outside samples)
    value[0, 6, 1] = np.nan         # on level 0's top border (5 x 7 map)
    value[1, 35, 0] = -np.inf       # level 1's first pixel
    g["value"] = value
    q = {k: (torch.from_numpy(v).to(dtype).float().numpy() if v.dtype == np.float32 else v) for k, v in g.items()}
    exp = oracle_forward(*[q[k] for k in INPUTS])
    inp = {k: torch.from_numpy(v).to(cuda_device) for k, v in q.items()}
    inp = {k: (v.to(dtype) if v.dtype.is_floating_point else v) for k, v in inp.items()}
    out = torch.empty(inp["grad_output"].shape, dtype=dtype, device=cuda_device)
    native.native_function("ms_deform_attn_forward")(*[inp[k] for k in INPUTS], out, 64)
    got = out.float().cpu()
    expected = torch.from_numpy(np.asarray(exp, dtype=np.float32))
    assert not torch.isfinite(expected).all()
    assert torch.equal(torch.isnan(got), torch.isnan(expected))
    assert torch.equal(torch.isinf(got), torch.isinf(expected))
    tol = FP32_TOL if dtype == torch.float32 else BF16_TOL
    fin = torch.isfinite(expected)
    torch.testing.assert_close(got[fin], expected[fin], rtol=tol, atol=tol)


def test_value_beyond_2_31_elements_indexes_every_image(cuda_device):
    """c2 shapes at 320 images (Lq 2000; a multiple of the im2col step): `value`
    holds 2.5e9 elements, so image 272 straddles 2^31 elements and image 319
    lies wholly past it, where a 32-bit offset anywhere in the kernels would
    read or write the wrong image. The batched call must equal each image run
    alone (forward, grad_loc and grad_w bit for bit; grad_value up to the order
    of its fp32 reductions)."""
    cfg = cases.CONFIGS["c2"].with_(batch=320, queries=2000)
    inp = cases.make_inputs(cfg, dtype=torch.bfloat16, device=cuda_device)
    assert inp["value"].numel() > 2**31
    out, (gv, gl, gw) = _c_abi_fwd_bwd(inp, torch.bfloat16)
    for b in (0, 272, 319):
        part = {k: (v[b : b + 1].contiguous() if k not in ("spatial_shapes", "level_start_index") else v)
                for k, v in inp.items()}
        o, (pgv, pgl, pgw) = _c_abi_fwd_bwd(part, torch.bfloat16)
        assert torch.equal(o, out[b : b + 1])
        assert torch.equal(pgl, gl[b : b + 1])
        assert torch.equal(pgw, gw[b : b + 1])
        torch.testing.assert_close(pgv, gv[b : b + 1], rtol=1e-5, atol=1e-5)

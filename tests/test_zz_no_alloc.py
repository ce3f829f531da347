"""msda_backward_static_scratch: the backward that allocates no device memory.

Runtimes that may not allocate GPU memory once they run (memory planned before
start-up, plugin hosts that own the device memory) call this entry point
instead of ms_deform_attn_backward / msda_backward. It works in one fixed
device array shared by every call, so it must give the regular backward's
gradients not only once but call after call, with the array still holding the
previous call's contents. This file runs last (its name sorts last), after
every other test, and also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from muspace_b200 import cases
from muspace_b200.runtime import native

pytestmark = pytest.mark.gpu

TOL = 1e-4  # fp32 gradient buffers on both sides; they differ only in the order of fp32 atomic adds
NAMES = ("value", "spatial_shapes", "level_start_index", "sampling_locations", "attention_weights")


class _Dims(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in ("batch", "spatial_size", "heads", "channels", "levels", "queries", "points")]


def _static_scratch_backward(inp, grad, dtype):
    lib = native.load_native_module().lib
    fn = lib.msda_backward_static_scratch
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int, ctypes.POINTER(_Dims)] + [ctypes.c_void_p] * 10
    value, loc = inp["value"], inp["sampling_locations"]
    dims = _Dims(value.shape[0], value.shape[1], value.shape[2], value.shape[3], loc.shape[3], loc.shape[1], loc.shape[4])
    gv = torch.zeros(value.shape, dtype=torch.float32, device=value.device)
    gl = torch.full(loc.shape, float("nan"), dtype=torch.float32, device=value.device)
    gw = torch.full(inp["attention_weights"].shape, float("nan"), dtype=torch.float32, device=value.device)
    ptrs = [inp[n].data_ptr() for n in NAMES] + [grad.data_ptr(), gv.data_ptr(), gl.data_ptr(), gw.data_ptr()]
    code = 1 if dtype == torch.bfloat16 else 0
    status = fn(code, ctypes.byref(dims), *ptrs, torch.cuda.current_stream(value.device).cuda_stream)
    assert status == 0, native.load_native_module().last_error()
    return gv, gl, gw


def _regular_backward(inp, grad):
    value, loc, weight = inp["value"], inp["sampling_locations"], inp["attention_weights"]
    gv = torch.zeros(value.shape, dtype=torch.float32, device=value.device)
    gl = torch.empty(loc.shape, dtype=torch.float32, device=value.device)
    gw = torch.empty(weight.shape, dtype=torch.float32, device=value.device)
    native.native_function("ms_deform_attn_backward")(*(inp[n] for n in NAMES), grad, gv, gl, gw, 64)
    return gv, gl, gw


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_static_scratch_backward_matches_the_regular_backward_on_consecutive_calls(cuda_device, dtype):
    # BEVFormer SCA shapes at two camera images: inside the static scratch limit
    cfg = cases.CONFIGS["c2"].with_(batch=2)
    for seed in (11, 12):  # two calls in a row, the second over the first one's scratch
        inp = cases.make_inputs(cfg, dtype=dtype, seed=seed, device=cuda_device)
        grad = inp["grad_output"].contiguous()
        got = _static_scratch_backward(inp, grad, dtype)
        want = _regular_backward(inp, grad)
        torch.cuda.synchronize()
        for name, g, w in zip(("grad_value", "grad_sampling_locations", "grad_attention_weights"), got, want):
            assert not torch.isnan(g).any(), f"{name} left unwritten (seed {seed})"
            torch.testing.assert_close(g, w, rtol=TOL, atol=TOL, msg=lambda m, name=name: f"seed {seed} {name}: {m}")

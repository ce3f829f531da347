"""msda_backward_static_scratch: the backward that allocates no device memory.

Runtimes that may not allocate GPU memory once they run (memory planned before
start-up, plugin hosts that own the device memory) call this entry point
instead of ms_deform_attn_backward / msda_backward. It works in one fixed
device array shared by every call, so it must give the regular backward's
gradients not only once but call after call, with the array still holding the
previous call's contents, and it must not allocate while it runs. This file
runs last (its name sorts last), after every other test, and also passes
alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import load_golden
from muspace_b200 import cases
from muspace_b200.runtime import native
from oracle import oracle_backward

pytestmark = pytest.mark.gpu

TOL = 1e-4  # fp32 gradient buffers on both sides; they differ only in the order of fp32 atomic adds
NAMES = ("value", "spatial_shapes", "level_start_index", "sampling_locations", "attention_weights")


class _Dims(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in ("batch", "spatial_size", "heads", "channels", "levels", "queries", "points")]


class _DriverMemory:
    """Device memory in use, from the CUDA driver: the default memory pool's
    high-water mark (what cudaMallocAsync draws from) and the device's free
    bytes (what cudaMalloc draws from)."""

    USED_MEM_CURRENT = 7  # CU_MEMPOOL_ATTR_USED_MEM_CURRENT
    USED_MEM_HIGH = 8  # CU_MEMPOOL_ATTR_USED_MEM_HIGH

    def __init__(self, device: torch.device):
        self.cu = ctypes.CDLL("libcuda.so.1")
        dev = ctypes.c_int()
        assert self.cu.cuDeviceGet(ctypes.byref(dev), device.index) == 0
        self.pool = ctypes.c_void_p()
        assert self.cu.cuDeviceGetDefaultMemPool(ctypes.byref(self.pool), dev) == 0

    def reset_pool_high(self) -> None:
        zero = ctypes.c_uint64(0)
        assert self.cu.cuMemPoolSetAttribute(self.pool, self.USED_MEM_HIGH, ctypes.byref(zero)) == 0

    def _pool(self, attr: int) -> int:
        value = ctypes.c_uint64()
        assert self.cu.cuMemPoolGetAttribute(self.pool, attr, ctypes.byref(value)) == 0
        return value.value

    def pool_high(self) -> int:
        return self._pool(self.USED_MEM_HIGH)

    def pool_used(self) -> int:
        return self._pool(self.USED_MEM_CURRENT)

    def free_bytes(self) -> int:
        free, total = ctypes.c_size_t(), ctypes.c_size_t()
        assert self.cu.cuMemGetInfo_v2(ctypes.byref(free), ctypes.byref(total)) == 0
        return free.value


def _buffers(inp):
    value, loc = inp["value"], inp["sampling_locations"]
    gv = torch.zeros(value.shape, dtype=torch.float32, device=value.device)
    gl = torch.full(loc.shape, float("nan"), dtype=torch.float32, device=value.device)
    gw = torch.full(inp["attention_weights"].shape, float("nan"), dtype=torch.float32, device=value.device)
    return gv, gl, gw


def _static_scratch_call(inp, grad, dtype, gv, gl, gw):
    lib = native.load_native_module().lib
    fn = lib.msda_backward_static_scratch
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int, ctypes.POINTER(_Dims)] + [ctypes.c_void_p] * 10
    value, loc = inp["value"], inp["sampling_locations"]
    dims = _Dims(value.shape[0], value.shape[1], value.shape[2], value.shape[3], loc.shape[3], loc.shape[1], loc.shape[4])
    ptrs = [inp[n].data_ptr() for n in NAMES] + [grad.data_ptr(), gv.data_ptr(), gl.data_ptr(), gw.data_ptr()]
    code = 1 if dtype == torch.bfloat16 else 0
    status = fn(code, ctypes.byref(dims), *ptrs, torch.cuda.current_stream(value.device).cuda_stream)
    assert status == 0, native.load_native_module().last_error()


def _static_scratch_backward(inp, grad, dtype):
    gv, gl, gw = _buffers(inp)
    _static_scratch_call(inp, grad, dtype, gv, gl, gw)
    return gv, gl, gw


def _regular_backward(inp, grad):
    value, loc, weight = inp["value"], inp["sampling_locations"], inp["attention_weights"]
    gv = torch.zeros(value.shape, dtype=torch.float32, device=value.device)
    gl = torch.empty(loc.shape, dtype=torch.float32, device=value.device)
    gw = torch.empty(weight.shape, dtype=torch.float32, device=value.device)
    native.native_function("ms_deform_attn_backward")(*(inp[n] for n in NAMES), grad, gv, gl, gw, 64)
    return gv, gl, gw


def _compare(got, want, tol, what):
    for name, g, w in zip(("grad_value", "grad_sampling_locations", "grad_attention_weights"), got, want):
        g = g.float().cpu() if torch.is_tensor(g) else torch.from_numpy(np.asarray(g))
        w = w.float().cpu() if torch.is_tensor(w) else torch.from_numpy(np.asarray(w))
        assert not torch.isnan(g).any(), f"{what}: {name} left unwritten"
        torch.testing.assert_close(g, w, rtol=tol, atol=tol, msg=lambda m, name=name: f"{what} {name}: {m}")


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
        _compare(got, want, TOL, f"seed {seed}")


@pytest.mark.parametrize("channels", [16, 64, 128, 5])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_static_scratch_backward_every_channel_layout(cuda_device, channels, dtype):
    """The bucketed scatter kernel's channel instantiations (D = 16, 64, 128
    next to the D = 32 above) and an odd D, for which no vector layout exists
    and the call runs the scratch-free scalar backward with no scratch at all;
    two calls in a row each."""
    cfg = cases.CONFIGS["c2"].with_(batch=2, queries=600, channels=channels, heads=4,
                                     shapes=((29, 50), (15, 25), (8, 13), (4, 7)))
    for seed in (21, 22):
        inp = cases.make_inputs(cfg, dtype=dtype, seed=seed, device=cuda_device)
        grad = inp["grad_output"].contiguous()
        got = _static_scratch_backward(inp, grad, dtype)
        want = _regular_backward(inp, grad)
        torch.cuda.synchronize()
        _compare(got, want, TOL, f"D={channels} seed {seed}")


@pytest.mark.parametrize("name", ["edges", "c4_small_oob", "all_oob"])
def test_static_scratch_backward_matches_the_oracle_on_edge_goldens(cuda_device, name):
    """Exact level borders, out-of-bounds locations and a case with every
    sample outside its level, against the C oracle (pinned to the reference's
    own golden vectors), twice in a row."""
    g = load_golden(name)
    args = [g[k] for k in NAMES]
    want = oracle_backward(*args, g["grad_output"])
    inp = {k: torch.from_numpy(g[k]).to(cuda_device) for k in NAMES}
    grad = torch.from_numpy(g["grad_output"]).to(cuda_device).contiguous()
    for call in range(2):
        got = _static_scratch_backward(inp, grad, torch.float32)
        torch.cuda.synchronize()
        _compare(got, want, TOL, f"{name} call {call}")


def test_static_scratch_backward_allocates_no_device_memory(cuda_device):
    """The entry point's promise itself: while a call runs, nothing is taken
    from the stream-ordered allocator (the default pool's high-water mark
    stays where it was), from cudaMalloc (the device's free bytes do not change)
    or from torch's caching allocator."""
    cfg = cases.CONFIGS["c2"].with_(batch=2)
    inp = cases.make_inputs(cfg, dtype=torch.bfloat16, seed=31, device=cuda_device)
    grad = inp["grad_output"].contiguous()
    gv, gl, gw = _buffers(inp)
    _static_scratch_call(inp, grad, torch.bfloat16, gv, gl, gw)  # first call on the device: sets up the address
    torch.cuda.synchronize()
    mem = _DriverMemory(cuda_device)
    for _ in range(2):
        gv.zero_()
        torch.cuda.synchronize()
        mem.reset_pool_high()  # the high-water mark restarts from the memory in use now
        used_before = mem.pool_used()
        free_before = mem.free_bytes()
        torch_before = torch.cuda.memory_allocated(cuda_device)
        _static_scratch_call(inp, grad, torch.bfloat16, gv, gl, gw)
        torch.cuda.synchronize()
        assert mem.pool_high() == used_before, "the call drew on the stream-ordered allocator"
        assert mem.free_bytes() == free_before, "device memory was allocated during the call"
        assert torch.cuda.memory_allocated(cuda_device) == torch_before

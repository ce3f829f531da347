"""Loader for ``muspace_b200/native/libmuspace_ops.so`` (the C-ABI of ``include/muspace_msda.h``).

Takes the place of muSPACE's TVM-FFI loader (``mu_space/runtime/native.py:20-77``):
the same names (``load_native_module``, ``native_function``,
``native_module_proxy``, ``native_available``, ``native_error``,
``NativeModuleUnavailable``) and the same error messages for a missing
library, a library that fails to load and a missing export. The binding is
``ctypes`` over plain C: every torch tensor argument is described to the
library as a DLPack ``DLTensor`` view (no copy, no torch types cross the
boundary) and the call is enqueued on the tensor device's current CUDA stream,
as the reference's ``TVMFFIEnvGetStream`` did. A non-zero status becomes a
``RuntimeError`` carrying ``msda_last_error()``.
"""

from __future__ import annotations

import ctypes
from functools import lru_cache
from importlib.resources import files
from pathlib import Path
from typing import Any, Callable

import torch

LIBRARY_NAME = "native/libmuspace_ops.so"


class NativeModuleUnavailable(RuntimeError):
    """The package does not contain a usable native library."""


# --------------------------------------------------------------------------------------
# DLPack views (ABI of include/muspace_msda.h)
# --------------------------------------------------------------------------------------

K_DL_CPU = 1
K_DL_CUDA = 2


class DLDevice(ctypes.Structure):
    _fields_ = [("device_type", ctypes.c_int32), ("device_id", ctypes.c_int32)]


class DLDataType(ctypes.Structure):
    _fields_ = [("code", ctypes.c_uint8), ("bits", ctypes.c_uint8), ("lanes", ctypes.c_uint16)]


class DLTensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("device", DLDevice),
        ("ndim", ctypes.c_int32),
        ("dtype", DLDataType),
        ("shape", ctypes.POINTER(ctypes.c_int64)),
        ("strides", ctypes.POINTER(ctypes.c_int64)),
        ("byte_offset", ctypes.c_uint64),
    ]


_DTYPE_CODES = {
    torch.float32: (2, 32),
    torch.float64: (2, 64),
    torch.float16: (2, 16),
    torch.bfloat16: (4, 16),
    torch.int64: (0, 64),
    torch.int32: (0, 32),
    torch.uint8: (1, 8),
}


class _View:
    """A DLTensor describing a tensor, plus the shape and stride arrays it points into."""

    __slots__ = ("shape", "strides", "dl")

    def __init__(self, tensor: torch.Tensor):
        if tensor.dtype not in _DTYPE_CODES:
            raise TypeError(f"unsupported tensor dtype {tensor.dtype}")
        ndim = tensor.dim()
        self.shape = (ctypes.c_int64 * max(ndim, 1))(*tensor.shape)
        self.strides = (ctypes.c_int64 * max(ndim, 1))(*tensor.stride())
        code, bits = _DTYPE_CODES[tensor.dtype]
        if tensor.device.type == "cuda":
            device = DLDevice(K_DL_CUDA, tensor.device.index if tensor.device.index is not None else 0)
        else:
            device = DLDevice(K_DL_CPU, 0)
        self.dl = DLTensor(
            ctypes.c_void_p(tensor.data_ptr() if tensor.numel() else 0),
            device,
            ndim,
            DLDataType(code, bits, 1),
            ctypes.cast(self.shape, ctypes.POINTER(ctypes.c_int64)),
            ctypes.cast(self.strides, ctypes.POINTER(ctypes.c_int64)),
            0,
        )


# Descriptors by (data pointer, dtype, device, shape, strides): every field of a
# DLTensor, so a hit describes the argument exactly even when the memory it was
# first built for has since been freed and handed to another tensor. Building a
# descriptor costs ~9 us of Python; a per-camera launch loop reuses the same few.
_VIEW_CACHE: dict[tuple, _View] = {}
_VIEW_CACHE_LIMIT = 1024


def _view_of(tensor: torch.Tensor) -> _View:
    key = (tensor.data_ptr(), tensor.dtype, tensor.device, tensor.shape, tensor.stride())
    view = _VIEW_CACHE.get(key)
    if view is None:
        if len(_VIEW_CACHE) >= _VIEW_CACHE_LIMIT:
            _VIEW_CACHE.clear()
        view = _VIEW_CACHE[key] = _View(tensor)
    return view


def _stream_of(tensors) -> int:
    for t in tensors:
        if isinstance(t, torch.Tensor) and t.device.type == "cuda":
            return torch.cuda.current_stream(t.device).cuda_stream
    return 0


# argument kinds of the DLPack entry points: "t" tensor, "i" int, "f" float (the stream is appended)
_SIGNATURES: dict[str, tuple[str, ...]] = {
    "ms_deform_attn_forward": ("t",) * 6 + ("i",),
    "ms_deform_attn_backward": ("t",) * 9 + ("i",),
    "ms_deform_attn_backward_deterministic": ("t",) * 10 + ("i",),
    "ms_deform_attn_scatter_div_forward": ("t",) * 8 + ("i",),
    "deformable_aggregation_forward_opt": ("t",) * 6,
    "deformable_aggregation_forward_base": ("t",) * 6,
    "deformable_aggregation_backward_opt": ("t",) * 9,
    "deformable_aggregation_backward_base": ("t",) * 9,
    # value .. out, num_heads, num_points, gx, gy, gz, voxel size xyz, voxel min xyz, value_stride_n, epsilon
    "flash_bevpool_sca_forward": ("t",) * 8 + ("i",) * 5 + ("f",) * 6 + ("i", "f"),
    # out_grad .. attention_weights_grad, num_heads, num_points, gx, gy, gz, value_stride_n, epsilon
    "flash_bevpool_sca_backward": ("t",) * 12 + ("i",) * 6 + ("f",),
}


class NativeModule:
    """The loaded library; ``get_function`` mirrors tvm_ffi's Module API."""

    def __init__(self, lib: ctypes.CDLL, path: Path):
        self.lib = lib
        self.path = path
        lib.msda_last_error.restype = ctypes.c_char_p
        lib.msda_last_error.argtypes = []
        lib.msda_version.restype = ctypes.c_char_p
        lib.msda_version.argtypes = []
        self._cache: dict[str, Callable[..., None]] = {}

    def last_error(self) -> str:
        return self.lib.msda_last_error().decode()

    def version(self) -> str:
        return self.lib.msda_version().decode()

    def get_function(self, name: str) -> Callable[..., None]:
        if name in self._cache:
            return self._cache[name]
        symbol = getattr(self.lib, name)  # AttributeError when not exported
        signature = _SIGNATURES.get(name)
        if signature is None:
            fn = symbol
        else:
            symbol.restype = ctypes.c_int
            kinds = {"t": ctypes.POINTER(DLTensor), "i": ctypes.c_int, "f": ctypes.c_float}
            symbol.argtypes = [kinds[kind] for kind in signature] + [ctypes.c_void_p]
            fn = self._tensor_call(name, symbol, signature)
        self._cache[name] = fn
        return fn

    def _tensor_call(self, name: str, symbol, signature: tuple[str, ...]) -> Callable[..., None]:
        def call(*args: Any) -> None:
            if len(args) != len(signature):
                raise TypeError(f"{name} takes {len(signature)} arguments, got {len(args)}")
            views = []
            c_args = []
            for kind, arg in zip(signature, args):
                if kind == "t":
                    if not isinstance(arg, torch.Tensor):
                        raise TypeError(f"{name}: expected a tensor, got {type(arg).__name__}")
                    view = _view_of(arg)
                    views.append(view)
                    c_args.append(ctypes.byref(view.dl))
                elif kind == "f":
                    c_args.append(float(arg))
                else:
                    c_args.append(int(arg))
            stream = _stream_of(args)
            status = symbol(*c_args, ctypes.c_void_p(stream))
            if status != 0:
                raise RuntimeError(f"{name}: {self.last_error()}")

        call.__name__ = name
        return call


@lru_cache(maxsize=1)
def load_native_module() -> NativeModule:
    library = Path(files("muspace_b200").joinpath(LIBRARY_NAME))
    if not library.is_file():
        raise NativeModuleUnavailable(
            "muSPACE-B200 native library is missing from this installation; "
            "build it with `python -m muspace_b200.build` (nvcc, sm_100a)."
        )
    try:
        return NativeModule(ctypes.CDLL(str(library)), library)
    except OSError as exc:
        raise NativeModuleUnavailable(f"unable to load muSPACE-B200 native library {library}: {exc}") from exc


def native_function(name: str) -> Callable[..., Any]:
    module = load_native_module()
    try:
        return module.get_function(name)
    except (AttributeError, KeyError) as exc:
        raise NativeModuleUnavailable(f"muSPACE-B200 native library does not export {name!r}") from exc


class MsdaDims(ctypes.Structure):
    """``msda_dims_t`` of include/muspace_msda.h."""

    _fields_ = [(name, ctypes.c_int64) for name in
                ("batch", "spatial_size", "heads", "channels", "levels", "queries", "points")]


def deterministic_workspace_bytes(batch: int, spatial_size: int, heads: int, channels: int, levels: int,
                                  queries: int, points: int) -> int:
    """``msda_deterministic_workspace_bytes``: device bytes the deterministic
    backward needs for these sizes."""
    module = load_native_module()
    fn = module.lib.msda_deterministic_workspace_bytes
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(MsdaDims), ctypes.POINTER(ctypes.c_size_t)]
    dims = MsdaDims(batch, spatial_size, heads, channels, levels, queries, points)
    out = ctypes.c_size_t(0)
    if fn(ctypes.byref(dims), ctypes.byref(out)) != 0:
        raise RuntimeError(f"msda_deterministic_workspace_bytes: {module.last_error()}")
    return int(out.value)


class NativeModuleProxy:
    """Attribute-compatible view used by the operator wrappers."""

    def __getattr__(self, name: str) -> Any:
        return native_function(name)


@lru_cache(maxsize=1)
def native_module_proxy() -> NativeModuleProxy:
    load_native_module()
    return NativeModuleProxy()


def native_available() -> bool:
    try:
        load_native_module()
    except NativeModuleUnavailable:
        return False
    return True


def native_error() -> str | None:
    try:
        load_native_module()
    except NativeModuleUnavailable as exc:
        return str(exc)
    return None

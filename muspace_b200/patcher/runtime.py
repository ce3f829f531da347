"""Runtime hook that routes OpenMMLab's MSDA helper to the B200 kernels.

Mirrors the MSDA part of ``mu_space/patcher/runtime.py`` in the reference
(constants 14-41, ``_MissingLegacyExtension`` 97-119, the mmcv ``_ext`` guard
122-160, ``_patch_attr`` / ``_restore_attrs`` 212-258, ``PatchReport`` 262-269,
``_env_strict`` 272-273, ``_make_msda_wrapper`` 398-439, ``DefaultPatcher``
577-637 and the ``default_patcher`` instance 2020): ``default_patcher.apply()``
rebinds ``mmcv.ops.multi_scale_deform_attn.multi_scale_deformable_attn_pytorch``
and the copies BEVFormer / UniAD modules imported before the call;
``restore()`` undoes every rebind and releases the ``_ext`` guard.

Strict mode (``apply(strict=True)`` or ``MUSPACE_STRICT_PATCH=1``) sends every
call to the CUDA kernels. Compat mode sends CUDA tensors to the kernels and
hands any other tensor back to the function it replaced (mmcv's own PyTorch
implementation), so CPU code paths of the model behave exactly as without the
patch; this build ships no CPU implementation of its own.
"""

from __future__ import annotations

import importlib
import os
import sys
from collections.abc import Callable
from dataclasses import asdict, dataclass
from types import ModuleType

PatchCallable = Callable[..., object]

STRICT_ENV = "MUSPACE_STRICT_PATCH"
MSDA_TARGET_MODULE = "mmcv.ops.multi_scale_deform_attn"
MSDA_TARGET_ATTR = "multi_scale_deformable_attn_pytorch"
BEVFORMER_IMPORTED_MODULES = (
    "projects.mmdet3d_plugin.bevformer.modules.decoder",
    "projects.mmdet3d_plugin.bevformer.modules.encoder",
    "projects.mmdet3d_plugin.bevformer.modules.spatial_cross_attention",
    "projects.mmdet3d_plugin.bevformer.modules.temporal_self_attention",
)
UNIAD_IMPORTED_MODULES = (
    "projects.mmdet3d_plugin.uniad.modules.decoder",
    "projects.mmdet3d_plugin.uniad.modules.spatial_cross_attention",
    "projects.mmdet3d_plugin.uniad.modules.temporal_self_attention",
    "projects.mmdet3d_plugin.uniad.dense_heads.motion_head_plugin.motion_deformable_attn",
)
_MISSING = object()


class PatchError(RuntimeError):
    """Raised when runtime patching cannot be installed safely."""


class _MissingLegacyExtension:
    """Stands in for an mmcv extension that failed to load during model imports.

    Attribute probes (``hasattr``) succeed; calling any function raises
    ``PatchError`` with the extension and function name.
    """

    def __init__(self, name: str, functions: object) -> None:
        self.name = name
        self.functions = functions

    def __getattr__(self, attr: str) -> object:
        if attr.startswith("__") and attr.endswith("__"):
            raise AttributeError(attr)
        if attr in {"get_compiler_version", "get_compiling_cuda_version"}:
            return lambda: "unavailable"

        def unavailable(*args: object, **kwargs: object) -> object:
            raise PatchError(
                f"Legacy extension mmcv.{self.name} is unavailable; "
                f"the muSPACE replacement must handle this path before {attr} is called"
            )

        unavailable.__name__ = attr
        return unavailable


def _guard_legacy_mmcv_extensions() -> bool:
    """Make ``mmcv.utils.ext_loader.load_ext`` return a placeholder instead of
    raising when mmcv's compiled ``_ext`` is absent. Returns True when this
    call installed the guard (the caller then owns releasing it)."""
    try:
        ext_loader = importlib.import_module("mmcv.utils.ext_loader")
    except ImportError:
        return False
    if hasattr(ext_loader, "_muspace_original_load_ext"):
        return False
    original = ext_loader.load_ext

    def guarded_load_ext(name: str, functions: object):
        try:
            return original(name, functions)
        except (ImportError, OSError):
            return _MissingLegacyExtension(name, functions)

    ext_loader._muspace_original_load_ext = original
    ext_loader.load_ext = guarded_load_ext
    return True


def _release_legacy_mmcv_extensions() -> bool:
    ext_loader = sys.modules.get("mmcv.utils.ext_loader")
    if ext_loader is None:
        return False
    original = getattr(ext_loader, "_muspace_original_load_ext", None)
    if original is None:
        return False
    ext_loader.load_ext = original
    del ext_loader._muspace_original_load_ext
    return True


def _patch_attr(originals: dict[tuple[str, str], object], module: ModuleType, attr: str, replacement: object) -> bool:
    """Rebind ``module.attr``, remembering the first value seen for ``restore()``."""
    if not hasattr(module, attr):
        return False
    key = (module.__name__, attr)
    if key not in originals:
        originals[key] = getattr(module, attr)
    setattr(module, attr, replacement)
    return True


def _restore_attrs(originals: dict[tuple[str, str], object]) -> list[str]:
    restored = []
    for (module_name, attr), original in list(originals.items()):
        module = sys.modules.get(module_name)
        if module is not None:
            if original is _MISSING:
                if hasattr(module, attr):
                    delattr(module, attr)
            else:
                setattr(module, attr, original)
            restored.append(module_name)
        del originals[(module_name, attr)]
    return restored


@dataclass(frozen=True)
class PatchReport:
    target: str
    strict: bool
    action: str
    patched_modules: tuple[str, ...]

    def as_dict(self) -> dict[str, object]:
        return asdict(self)


def _env_strict() -> bool:
    return os.environ.get(STRICT_ENV, "").strip().lower() in {"1", "true", "yes", "on"}


def _level_start_index(value_spatial_shapes):
    import torch

    level_sizes = value_spatial_shapes[:, 0] * value_spatial_shapes[:, 1]
    if level_sizes.numel() == 0:
        return level_sizes.new_empty(0)
    return torch.cat([level_sizes.new_zeros(1), level_sizes.cumsum(0)[:-1]])


def _is_cuda(value) -> bool:
    return getattr(getattr(value, "device", None), "type", None) == "cuda"


def _make_msda_wrapper(strict: bool, original: PatchCallable | None = None) -> PatchCallable:
    if strict:

        def strict_msda(value, value_spatial_shapes, sampling_locations, attention_weights):
            from muspace_b200.ops import multi_scale_deformable_attn

            return multi_scale_deformable_attn(
                value,
                value_spatial_shapes,
                _level_start_index(value_spatial_shapes),
                sampling_locations,
                attention_weights,
                backend="cuda",
            )

        strict_msda.__name__ = "muspace_multi_scale_deformable_attn_strict"
        strict_msda.__module__ = __name__
        return strict_msda

    def compat_msda(value, value_spatial_shapes, sampling_locations, attention_weights):
        if not _is_cuda(value) and original is not None:
            return original(value, value_spatial_shapes, sampling_locations, attention_weights)
        from muspace_b200.ops import multi_scale_deformable_attn_pytorch_compat

        return multi_scale_deformable_attn_pytorch_compat(
            value, value_spatial_shapes, sampling_locations, attention_weights
        )

    compat_msda.__name__ = "muspace_multi_scale_deformable_attn_compat"
    compat_msda.__module__ = __name__
    return compat_msda


class DefaultPatcher:
    """Install the MSDA runtime patch without editing user model code."""

    def __init__(self) -> None:
        self._originals: dict[tuple[str, str], object] = {}
        self._strict: bool | None = None
        self._guarded = False

    def apply(self, *, strict: bool | None = None) -> PatchReport:
        strict = _env_strict() if strict is None else strict
        patched_modules = self._patch_mmcv_msda(strict)
        action = "already-applied" if self._strict == strict else "applied"
        self._strict = strict
        return PatchReport(
            target=f"{MSDA_TARGET_MODULE}.{MSDA_TARGET_ATTR}",
            strict=strict,
            action=action,
            patched_modules=tuple(patched_modules),
        )

    def restore(self) -> PatchReport:
        restored = _restore_attrs(self._originals)
        if self._guarded:
            _release_legacy_mmcv_extensions()
            self._guarded = False
        self._strict = None
        return PatchReport(
            target=f"{MSDA_TARGET_MODULE}.{MSDA_TARGET_ATTR}",
            strict=False,
            action="restored",
            patched_modules=tuple(restored),
        )

    def _patch_attr(self, module: ModuleType, attr: str, replacement: object) -> bool:
        return _patch_attr(self._originals, module, attr, replacement)

    def _patch_mmcv_msda(self, strict: bool) -> list[str]:
        self._guarded = _guard_legacy_mmcv_extensions() or self._guarded
        try:
            target = importlib.import_module(MSDA_TARGET_MODULE)
        except ImportError as exc:
            raise PatchError(
                "mmcv MSDeformAttn helper is unavailable; install the BEVFormer "
                "OpenMMLab stack before calling default_patcher.apply()"
            ) from exc
        if not hasattr(target, MSDA_TARGET_ATTR):
            raise PatchError(f"{MSDA_TARGET_MODULE}.{MSDA_TARGET_ATTR} is unavailable")
        # the function mmcv shipped, even when apply() runs twice
        original = self._originals.get((target.__name__, MSDA_TARGET_ATTR), getattr(target, MSDA_TARGET_ATTR))
        replacement = _make_msda_wrapper(strict, original)
        patched = []
        self._patch_attr(target, MSDA_TARGET_ATTR, replacement)
        patched.append(target.__name__)
        # model modules bind the helper at import time; rebind those globals too
        for module_name in (*BEVFORMER_IMPORTED_MODULES, *UNIAD_IMPORTED_MODULES):
            module = sys.modules.get(module_name)
            if module is not None and self._patch_attr(module, MSDA_TARGET_ATTR, replacement):
                patched.append(module_name)
        return patched


# Qwen-Drive's perception head (patcher/runtime.py:77-81 of the reference)
QWENDRIVE_ATTENTION_MODULE = "qwen_drive_perception.attention"
QWENDRIVE_MSDA_ATTR = "multi_scale_deformable_attn_cuda"
QWENDRIVE_OPS_MODULE = "qwen_drive_perception.ops"
QWENDRIVE_MSDA_FORWARD_ATTR = "ms_deform_attn_bf16_forward"


def _make_qwendrive_msda_wrapper(strict: bool, original: PatchCallable) -> PatchCallable:
    """Six-argument Qwen-Drive MSDA entry (reference ``patcher/runtime.py:285-337``).

    Qwen-Drive calls ``(value, spatial_shapes, level_start_index, locations,
    weights, im2col_step)`` and its own kernel is bfloat16-only and forward-only.
    CUDA tensors go through the native autograd operator (forward and
    backward); a CUDA tensor that is not bfloat16 raises, as Qwen-Drive's gate
    does; anything else keeps Qwen-Drive's original function.
    """

    backend = "cuda" if strict else "auto"

    def muspace_qwendrive_msda(value, value_spatial_shapes, value_level_start_index, sampling_locations,
                               attention_weights, im2col_step):
        if not _is_cuda(value):
            return original(value, value_spatial_shapes, value_level_start_index, sampling_locations,
                            attention_weights, im2col_step)
        import torch

        if value.dtype != torch.bfloat16:
            raise TypeError(
                "the ms_deform_attn kernel requires bfloat16 tensors on CUDA, "
                f"got {value.dtype}; run the model in bfloat16"
            )
        from muspace_b200.ops import multi_scale_deformable_attn

        return multi_scale_deformable_attn(value, value_spatial_shapes, value_level_start_index, sampling_locations,
                                           attention_weights, im2col_step=int(im2col_step), backend=backend)

    muspace_qwendrive_msda.__name__ = "muspace_qwendrive_msda_strict" if strict else "muspace_qwendrive_msda"
    muspace_qwendrive_msda.__module__ = __name__
    return muspace_qwendrive_msda


class QwenDrivePatcher:
    """Route Qwen-Drive's multi-scale deformable attention onto the B200 operator.

    Reference: ``QwenDrivePatcher`` (``patcher/runtime.py:1897-2018``). It rebinds
    ``qwen_drive_perception.attention.multi_scale_deformable_attn_cuda`` and
    ``qwen_drive_perception.ops.ms_deform_attn_bf16_forward`` to one wrapper,
    which adds the backward Qwen-Drive's forward-only kernel lacks. The
    reference also replaces ``ops.voxel_pool_depth`` and the view transform's
    ``frustum`` property because Qwen-Drive's CUDA code cannot run on MUSA; on
    a CUDA GPU that code runs as shipped, so this patcher leaves both alone.
    """

    def __init__(self) -> None:
        self._originals: dict[tuple[str, str], object] = {}
        self._strict: bool | None = None

    def apply(self, *, strict: bool | None = None) -> PatchReport:
        strict = _env_strict() if strict is None else strict
        attention, ops = self._import_package()
        missing = [f"{QWENDRIVE_ATTENTION_MODULE}.{QWENDRIVE_MSDA_ATTR}"] if not callable(
            getattr(attention, QWENDRIVE_MSDA_ATTR, None)) else []
        if not callable(getattr(ops, QWENDRIVE_MSDA_FORWARD_ATTR, None)):
            missing.append(f"{QWENDRIVE_OPS_MODULE}.{QWENDRIVE_MSDA_FORWARD_ATTR}")
        if missing:
            raise PatchError(
                "qwen_drive_perception is missing the symbols this patcher replaces: " + ", ".join(missing)
            )
        # a second apply keeps Qwen-Drive's own function as the fallback
        original = self._originals.get((attention.__name__, QWENDRIVE_MSDA_ATTR),
                                       getattr(attention, QWENDRIVE_MSDA_ATTR))
        wrapper = _make_qwendrive_msda_wrapper(strict, original)
        patched = []
        if _patch_attr(self._originals, attention, QWENDRIVE_MSDA_ATTR, wrapper):
            patched.append(attention.__name__)
        if _patch_attr(self._originals, ops, QWENDRIVE_MSDA_FORWARD_ATTR, wrapper):
            patched.append(ops.__name__)
        action = "already-applied" if self._strict == strict else "applied"
        self._strict = strict
        return PatchReport(target=f"{QWENDRIVE_ATTENTION_MODULE}.{QWENDRIVE_MSDA_ATTR}", strict=strict,
                           action=action, patched_modules=tuple(patched))

    def restore(self) -> PatchReport:
        restored = _restore_attrs(self._originals)
        self._strict = None
        return PatchReport(target=f"{QWENDRIVE_ATTENTION_MODULE}.{QWENDRIVE_MSDA_ATTR}", strict=False,
                           action="restored", patched_modules=tuple(restored))

    @staticmethod
    def _import_package() -> tuple[ModuleType, ModuleType]:
        try:
            attention = importlib.import_module(QWENDRIVE_ATTENTION_MODULE)
            ops = importlib.import_module(QWENDRIVE_OPS_MODULE)
        except ImportError as exc:
            raise PatchError(
                "qwen_drive_perception import failed. Add the Qwen-Drive checkout src "
                "directory to PYTHONPATH before qwendrive_patcher.apply()."
            ) from exc
        return attention, ops


# SparseDrive's deformable aggregation (patcher/runtime.py:61-70 of the reference)
SPARSEDRIVE_OPS_MODULE = "projects.mmdet3d_plugin.ops"
SPARSEDRIVE_DAF_ATTR = "deformable_aggregation_function"
SPARSEDRIVE_IMPORTED_MODULES = ("projects.mmdet3d_plugin.models.blocks",)
SPARSEDRIVE_IMPORTED_ATTR = "DAF"
SPARSEDRIVE_PACKAGE = "projects"
SPARSEDRIVE_DAF_VALID_ATTR = "DAF_VALID"
SPARSEDRIVE_FEATURE_MAPS_ATTR = "feature_maps_format"
SPARSEDRIVE_EXT_MODULE = "projects.mmdet3d_plugin.ops.deformable_aggregation_ext"
SPARSEDRIVE_EXT_ATTR = "deformable_aggregation_ext"


def _make_deformable_aggregation_wrapper(strict: bool) -> PatchCallable:
    """SparseDrive's five-argument DAF entry (reference ``patcher/runtime.py:519-546``)."""
    backend = "cuda" if strict else "auto"

    def muspace_deformable_aggregation(feature_maps, spatial_shape, scale_start_index, sampling_location, weights):
        from muspace_b200.ops import deformable_aggregation_function

        return deformable_aggregation_function(feature_maps, spatial_shape, scale_start_index, sampling_location,
                                               weights, backend=backend)

    muspace_deformable_aggregation.__name__ = (
        "muspace_deformable_aggregation_strict" if strict else "muspace_deformable_aggregation_compat"
    )
    muspace_deformable_aggregation.__module__ = __name__
    return muspace_deformable_aggregation


class _MissingSparseDriveExtension(ModuleType):
    """Stands in for SparseDrive's unbuilt CUDA extension so its ops package
    imports; every use of it raises (the patched entry point never reaches it)."""

    def __getattr__(self, attr: str) -> object:
        if attr.startswith("__"):
            raise AttributeError(attr)
        raise PatchError(
            f"SparseDrive extension {SPARSEDRIVE_EXT_MODULE} is unavailable; the muSPACE-B200 "
            "runtime patch routes deformable aggregation to its own kernels"
        )


class SparseDrivePatcher:
    """Route SparseDrive's deformable aggregation onto the B200 operator.

    Reference: ``SparseDrivePatcher`` (``patcher/runtime.py:1292-1520``), DAF part:
    rebinds ``projects.mmdet3d_plugin.ops.deformable_aggregation_function`` and
    the ``DAF`` global of ``projects.mmdet3d_plugin.models.blocks``, lets the ops
    package import when its CUDA extension was never built, and flips the
    ``DAF_VALID`` flags that modules cached while the extension was missing. The
    reference's MATE / flash-attention bridge and its ``Tensor.cuda`` shim exist
    because SparseDrive's CUDA code cannot run on MUSA; on a CUDA GPU it runs as
    shipped, so this patcher leaves them alone.
    """

    def __init__(self) -> None:
        self._originals: dict[tuple[str, str], object] = {}
        self._strict: bool | None = None
        self._placeholder: ModuleType | None = None

    def apply(self, *, strict: bool | None = None) -> PatchReport:
        strict = _env_strict() if strict is None else strict
        wrapper = _make_deformable_aggregation_wrapper(strict)
        target = self._import_ops()
        try:
            if not self._patch(target, SPARSEDRIVE_DAF_ATTR, wrapper):
                raise PatchError(f"{SPARSEDRIVE_OPS_MODULE}.{SPARSEDRIVE_DAF_ATTR} is unavailable")
            patched = [target.__name__]
            for module_name in SPARSEDRIVE_IMPORTED_MODULES:
                module = sys.modules.get(module_name)
                if module is not None and self._patch(module, SPARSEDRIVE_IMPORTED_ATTR, wrapper):
                    patched.append(module_name)
            # modules that probed the ops import before it worked cached DAF_VALID = False
            prefix = f"{SPARSEDRIVE_PACKAGE}."
            for name, module in list(sys.modules.items()):
                if module is None or not (name == SPARSEDRIVE_PACKAGE or name.startswith(prefix)):
                    continue
                if getattr(module, SPARSEDRIVE_DAF_VALID_ATTR, None) is not False:
                    continue
                self._bind(module, SPARSEDRIVE_DAF_VALID_ATTR, True)
                fmt = getattr(target, SPARSEDRIVE_FEATURE_MAPS_ATTR, None)
                if fmt is not None and not hasattr(module, SPARSEDRIVE_FEATURE_MAPS_ATTR):
                    self._bind(module, SPARSEDRIVE_FEATURE_MAPS_ATTR, fmt)
                patched.append(name)
        except BaseException:
            _restore_attrs(self._originals)
            self._release_placeholder()
            raise
        action = "already-applied" if self._strict == strict else "applied"
        self._strict = strict
        return PatchReport(target=f"{SPARSEDRIVE_OPS_MODULE}.{SPARSEDRIVE_DAF_ATTR}", strict=strict, action=action,
                           patched_modules=tuple(patched))

    def restore(self) -> PatchReport:
        restored = _restore_attrs(self._originals)
        self._release_placeholder()
        self._strict = None
        return PatchReport(target=f"{SPARSEDRIVE_OPS_MODULE}.{SPARSEDRIVE_DAF_ATTR}", strict=False,
                           action="restored", patched_modules=tuple(restored))

    def _patch(self, module: ModuleType, attr: str, replacement: object) -> bool:
        return _patch_attr(self._originals, module, attr, replacement)

    def _bind(self, module: ModuleType, attr: str, value: object) -> None:
        """Set an attribute that may not exist yet; restore() deletes it again."""
        key = (module.__name__, attr)
        if key not in self._originals:
            self._originals[key] = getattr(module, attr, _MISSING)
        setattr(module, attr, value)

    def _import_ops(self) -> ModuleType:
        try:
            return importlib.import_module(SPARSEDRIVE_OPS_MODULE)
        except ImportError as exc:
            missing = getattr(exc, "name", None) in {SPARSEDRIVE_EXT_MODULE, SPARSEDRIVE_EXT_ATTR} or (
                SPARSEDRIVE_EXT_ATTR in str(exc))
            if not missing:
                raise PatchError(
                    "SparseDrive ops package import failed. Ensure the SparseDrive checkout is on PYTHONPATH "
                    f"({exc})"
                ) from exc
        if SPARSEDRIVE_EXT_MODULE not in sys.modules:
            self._placeholder = _MissingSparseDriveExtension(SPARSEDRIVE_EXT_MODULE)
            sys.modules[SPARSEDRIVE_EXT_MODULE] = self._placeholder
        try:
            return importlib.import_module(SPARSEDRIVE_OPS_MODULE)
        except ImportError as exc:
            self._release_placeholder()
            raise PatchError(
                f"SparseDrive ops package import failed. Ensure the SparseDrive checkout is on PYTHONPATH ({exc})"
            ) from exc

    def _release_placeholder(self) -> None:
        placeholder, self._placeholder = self._placeholder, None
        if placeholder is not None and sys.modules.get(SPARSEDRIVE_EXT_MODULE) is placeholder:
            del sys.modules[SPARSEDRIVE_EXT_MODULE]


default_patcher = DefaultPatcher()
qwendrive_patcher = QwenDrivePatcher()
sparsedrive_patcher = SparseDrivePatcher()

__all__ = [
    "DefaultPatcher",
    "PatchError",
    "PatchReport",
    "QwenDrivePatcher",
    "SparseDrivePatcher",
    "default_patcher",
    "qwendrive_patcher",
    "sparsedrive_patcher",
]

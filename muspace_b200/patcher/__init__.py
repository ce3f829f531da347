"""Runtime patch entry points (the hooks of the reference's patcher on the
ops this build covers: mmcv's MSDA helper for BEVFormer / UniAD, Qwen-Drive's
MSDA entry and SparseDrive's deformable aggregation)."""

from .runtime import (
    DefaultPatcher,
    PatchError,
    PatchReport,
    QwenDrivePatcher,
    SparseDrivePatcher,
    default_patcher,
    qwendrive_patcher,
    sparsedrive_patcher,
)

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

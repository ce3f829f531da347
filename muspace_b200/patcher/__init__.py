"""Runtime patch entry points (the MSDA hooks of the reference's patcher:
mmcv's helper for BEVFormer / UniAD, and Qwen-Drive's MSDA entry)."""

from .runtime import DefaultPatcher, PatchError, PatchReport, QwenDrivePatcher, default_patcher, qwendrive_patcher

__all__ = ["DefaultPatcher", "PatchError", "PatchReport", "QwenDrivePatcher", "default_patcher", "qwendrive_patcher"]

"""Runtime patch entry points (the MSDA hook of the reference's patcher)."""

from .runtime import DefaultPatcher, PatchError, PatchReport, default_patcher

__all__ = ["DefaultPatcher", "PatchError", "PatchReport", "default_patcher"]

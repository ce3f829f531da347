"""Canonical operator exports of the B200 build (the MSDA operator)."""

from .multi_scale_deformable_attn import (
    explain_dispatch,
    multi_scale_deformable_attn,
    multi_scale_deformable_attn_pytorch_compat,
)

__all__ = [
    "explain_dispatch",
    "multi_scale_deformable_attn",
    "multi_scale_deformable_attn_pytorch_compat",
]

"""Canonical operator exports of the B200 build (the MSDA operator and the
fused spatial-cross-attention scatter built on it)."""

from .multi_scale_deformable_attn import (
    explain_dispatch,
    multi_scale_deformable_attn,
    multi_scale_deformable_attn_pytorch_compat,
)
from .sca_scatter import ms_deform_attn_scatter_div, sca_rebatch_scatter

__all__ = [
    "explain_dispatch",
    "ms_deform_attn_scatter_div",
    "multi_scale_deformable_attn",
    "multi_scale_deformable_attn_pytorch_compat",
    "sca_rebatch_scatter",
]

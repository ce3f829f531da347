"""Canonical operator exports of the B200 build: the MSDA operator, the fused
spatial-cross-attention scatter built on it, FlashSCA, and SparseDrive's
deformable aggregation."""

from .deformable_aggregation import (
    deformable_aggregation,
    deformable_aggregation_function,
    feature_maps_format,
)
from .multi_scale_deformable_attn import (
    explain_dispatch,
    multi_scale_deformable_attn,
    multi_scale_deformable_attn_pytorch_compat,
)
from .flash_sca import flash_bevpool_sca
from .sca_scatter import ms_deform_attn_scatter_div, sca_rebatch_scatter

__all__ = [
    "deformable_aggregation",
    "deformable_aggregation_function",
    "explain_dispatch",
    "feature_maps_format",
    "flash_bevpool_sca",
    "ms_deform_attn_scatter_div",
    "multi_scale_deformable_attn",
    "multi_scale_deformable_attn_pytorch_compat",
    "sca_rebatch_scatter",
]

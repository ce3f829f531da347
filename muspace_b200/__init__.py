"""muSPACE-B200: the multi-scale deformable attention path of muSPACE on NVIDIA B200.

The public names are those of the reference's ``mu_space`` package that belong
to the MSDA operator; ``import mu_space`` resolves to this package too.
"""

from .ops import explain_dispatch, multi_scale_deformable_attn, multi_scale_deformable_attn_pytorch_compat
from .runtime.kernel_dispatch import (
    DispatchDecision,
    DispatchReport,
    clear_dispatch_report,
    get_dispatch_reports,
    get_last_dispatch_report,
)

__version__ = "0.1.0"

__all__ = [
    "DispatchDecision",
    "DispatchReport",
    "__version__",
    "clear_dispatch_report",
    "explain_dispatch",
    "get_dispatch_reports",
    "get_last_dispatch_report",
    "multi_scale_deformable_attn",
    "multi_scale_deformable_attn_pytorch_compat",
]

"""Backend decision and dispatch reports for the B200 MSDA operator.

Mirrors ``mu_space/runtime/kernel_dispatch.py:13-103`` of the reference: the
same ``DispatchDecision`` / ``DispatchReport`` records, the same global report
log (``record_dispatch_report``, ``get_last_dispatch_report``,
``get_dispatch_reports``, ``clear_dispatch_report``) and the same
``MUSPACE_DISPATCH_LOG`` stderr JSON switch.

The decision itself is GPU-only. There is exactly one backend, the CUDA
kernels of ``libmuspace_ops.so``; ``backend="cuda"`` forces it and
``backend="musa"`` is accepted as the reference's spelling of "the native
backend", so code and patches written for muSPACE keep working. The
reference's ``backend="reference"`` (its PyTorch ``grid_sample`` path) and its
automatic CPU fallback are not part of this build: such requests are decided
``"error"`` with the reason, and nothing is ever silently computed on the CPU.
"""

from __future__ import annotations

import json
import os
import sys
from dataclasses import asdict, dataclass
from typing import Literal

import torch

BackendName = Literal["auto", "cuda", "musa"]
SelectedBackend = Literal["cuda", "error"]
NATIVE_BACKENDS = ("cuda", "musa")


@dataclass(frozen=True)
class DispatchDecision:
    backend: SelectedBackend
    device: str
    reason: str

    def as_dict(self) -> dict[str, object]:
        return asdict(self)


@dataclass(frozen=True)
class DispatchReport:
    operator: str
    requested_backend: str
    selected_backend: SelectedBackend
    device: str
    reason: str
    native_available: bool
    native_fallback: bool = False
    fallback_reason: str | None = None

    def as_dict(self) -> dict[str, object]:
        return asdict(self)


_last_dispatch_report: DispatchReport | None = None
_dispatch_reports: list[DispatchReport] = []


def record_dispatch_report(report: DispatchReport) -> DispatchReport:
    global _last_dispatch_report
    _last_dispatch_report = report
    _dispatch_reports.append(report)
    if os.environ.get("MUSPACE_DISPATCH_LOG", "").strip().lower() in {"1", "true", "yes", "on"}:
        print("muSPACE dispatch: " + json.dumps(report.as_dict(), sort_keys=True), file=sys.stderr)
    return report


def get_last_dispatch_report() -> DispatchReport | None:
    return _last_dispatch_report


def get_dispatch_reports() -> tuple[DispatchReport, ...]:
    return tuple(_dispatch_reports)


def clear_dispatch_report() -> None:
    global _last_dispatch_report, _dispatch_reports
    _last_dispatch_report = None
    _dispatch_reports = []


def _is_cuda_tensor(tensor: torch.Tensor) -> bool:
    return tensor.device.type == "cuda"


_KERNEL_NAMES = {"multi_scale_deformable_attn": "MSDA", "deformable_aggregation": "deformable aggregation",
                 "flash_bevpool_sca": "FlashSCA"}


def explain_dispatch(
    value: torch.Tensor,
    *,
    backend: str = "auto",
    native_available: bool = True,
    operator: str = "multi_scale_deformable_attn",
) -> DispatchDecision:
    device = value.device.type
    if backend == "reference":
        return DispatchDecision(
            "error",
            device,
            "the reference PyTorch backend is not part of the B200 build; "
            f"{operator} runs on CUDA tensors only",
        )
    if backend not in {"auto", *NATIVE_BACKENDS}:
        return DispatchDecision("error", device, f"unknown backend: {backend}")
    if not _is_cuda_tensor(value):
        kernels = _KERNEL_NAMES.get(operator, operator)
        return DispatchDecision(
            "error", device, f"the B200 {kernels} kernels need CUDA tensors; value is on {device}"
        )
    if not native_available:
        return DispatchDecision("error", device, "muSPACE-B200 native library is unavailable")
    if backend == "auto":
        return DispatchDecision("cuda", device, "CUDA tensor selects the native backend")
    return DispatchDecision("cuda", device, f"forced native backend ({backend})")

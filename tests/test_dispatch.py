"""Host-side behaviour of the canonical op on CPU: normalisation, GPU-only
dispatch and the dispatch report.

Follows the reference's CPU tests (``tests/ops/test_multi_scale_deformable_attn.py``
84-253, 471-481), retargeted: where the reference ran its PyTorch path on CPU
tensors, the B200 build must refuse loudly and record why.
"""

from __future__ import annotations

from importlib import import_module

import pytest
import torch

from mu_space import clear_dispatch_report, explain_dispatch, get_last_dispatch_report, multi_scale_deformable_attn

msda_module = import_module("mu_space.ops.multi_scale_deformable_attn")


def _fixture(dtype=torch.float32, *, batch=1, queries=5, heads=2, embed_dims=3, levels=((2, 2),), points=4):
    generator = torch.Generator(device="cpu").manual_seed(20260714)
    value_length = sum(h * w for h, w in levels)
    value = torch.randn(batch, value_length, heads, embed_dims, generator=generator, dtype=dtype)
    spatial_shapes = torch.tensor(levels, dtype=torch.int64)
    sizes = spatial_shapes[:, 0] * spatial_shapes[:, 1]
    level_start_index = torch.cat([sizes.new_zeros(1), sizes.cumsum(0)[:-1]])
    loc = torch.rand(batch, queries, heads, len(levels), points, 2, generator=generator, dtype=dtype)
    weights = torch.softmax(torch.rand(batch, queries, heads, len(levels), points, generator=generator, dtype=dtype), -1)
    return value, spatial_shapes, level_start_index, loc, weights


def test_cpu_tensors_are_refused_and_reported():
    clear_dispatch_report()
    with pytest.raises(RuntimeError, match="need CUDA tensors; value is on cpu"):
        multi_scale_deformable_attn(*_fixture())
    report = get_last_dispatch_report()
    assert report is not None
    assert report.operator == "multi_scale_deformable_attn"
    assert report.requested_backend == "auto"
    assert report.selected_backend == "error"
    assert report.native_fallback is False


def test_auto_cpu_dispatch_is_an_error_not_a_fallback():
    value, *_ = _fixture()
    decision = explain_dispatch(value, backend="auto")
    assert decision.backend == "error"
    assert decision.device == "cpu"


def test_reference_backend_is_not_part_of_the_build():
    clear_dispatch_report()
    with pytest.raises(RuntimeError, match="reference PyTorch backend is not part of the B200 build"):
        multi_scale_deformable_attn(*_fixture(), backend="reference")
    assert get_last_dispatch_report().selected_backend == "error"


def test_invalid_backend_fails_explicitly():
    clear_dispatch_report()
    with pytest.raises(RuntimeError, match="unknown backend"):
        multi_scale_deformable_attn(*_fixture(), backend="unknown")
    report = get_last_dispatch_report()
    assert report.selected_backend == "error"
    assert report.reason == "unknown backend: unknown"


def test_musa_spelling_selects_the_native_backend_for_cuda_tensors(monkeypatch):
    dispatch = import_module("mu_space.runtime.kernel_dispatch")
    fake = torch.empty(0)
    monkeypatch.setattr(dispatch, "_is_cuda_tensor", lambda t: True)
    for backend in ("musa", "cuda", "auto"):
        decision = dispatch.explain_dispatch(fake, backend=backend, native_available=True)
        assert decision.backend == "cuda", backend
    decision = dispatch.explain_dispatch(fake, backend="cuda", native_available=False)
    assert decision.backend == "error"
    assert "unavailable" in decision.reason


def test_dispatch_log_env_writes_stderr(monkeypatch, capsys):
    clear_dispatch_report()
    monkeypatch.setenv("MUSPACE_DISPATCH_LOG", "1")
    with pytest.raises(RuntimeError):
        multi_scale_deformable_attn(*_fixture())
    captured = capsys.readouterr()
    assert "muSPACE dispatch:" in captured.err
    assert '"selected_backend": "error"' in captured.err


def test_native_failure_raises_without_fallback(monkeypatch):
    """The reference's auto mode reran its PyTorch path after a native failure
    (test 204-229); this build records the error and re-raises it."""
    clear_dispatch_report()
    monkeypatch.setattr(msda_module, "_native_extension", lambda: object())
    monkeypatch.setattr(
        msda_module,
        "_explain_dispatch",
        lambda value, *, backend, native_available: msda_module.DispatchDecision(
            "cuda", value.device.type, "simulated CUDA tensor"
        ),
    )

    def fail_native(*args, **kwargs):
        raise RuntimeError("simulated native failure")

    monkeypatch.setattr(msda_module._NativeMSDAFunction, "apply", fail_native)
    with pytest.raises(RuntimeError, match="simulated native failure"):
        multi_scale_deformable_attn(*_fixture(), backend="auto")
    report = get_last_dispatch_report()
    assert report.selected_backend == "error"
    assert report.native_available is True
    assert report.native_fallback is False
    assert report.reason == "simulated native failure"


def test_spatial_shape_dtype_is_validated():
    value, spatial_shapes, start, loc, weights = _fixture()
    with pytest.raises(TypeError, match="spatial_shapes must be int64"):
        multi_scale_deformable_attn(value, spatial_shapes.to(torch.int32), start, loc, weights)


def test_level_start_index_dtype_is_validated():
    value, spatial_shapes, start, loc, weights = _fixture()
    with pytest.raises(TypeError, match="level_start_index must be int64"):
        multi_scale_deformable_attn(value, spatial_shapes, start.to(torch.int32), loc, weights)


def test_float64_value_is_rejected():
    value, spatial_shapes, start, loc, weights = _fixture()
    with pytest.raises(TypeError, match="value must be float16, bfloat16 or float32"):
        multi_scale_deformable_attn(value.double(), spatial_shapes, start, loc.double(), weights.double())


def test_sampling_and_attention_dtypes_follow_value_dtype():
    value, spatial_shapes, start, loc, weights = _fixture()
    normalized = msda_module._normalize_inputs(value, spatial_shapes, start, loc.double(), weights.double())
    assert normalized[3].dtype == value.dtype
    assert normalized[4].dtype == value.dtype
    assert all(t.is_contiguous() for t in normalized)


def test_normalize_makes_noncontiguous_inputs_contiguous():
    value, spatial_shapes, start, loc, weights = _fixture(batch=2, queries=3, heads=2, embed_dims=4)
    value_nc = torch.randn(*value.shape, 2)[..., 0]
    loc_nc = torch.rand(*loc.shape, 2)[..., 0]
    assert not value_nc.is_contiguous() and not loc_nc.is_contiguous()
    normalized = msda_module._normalize_inputs(value_nc, spatial_shapes, start, loc_nc, weights)
    assert all(t.is_contiguous() for t in normalized)
    torch.testing.assert_close(normalized[0], value_nc)

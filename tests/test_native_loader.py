"""Loader error messages (reference ``tests/test_native_loader.py:9-51``)."""

from __future__ import annotations

import pytest

from mu_space.runtime import native


@pytest.fixture(autouse=True)
def _fresh_loader():
    native.load_native_module.cache_clear()
    native.native_module_proxy.cache_clear()
    yield
    native.load_native_module.cache_clear()
    native.native_module_proxy.cache_clear()


def test_missing_library_is_explained(monkeypatch):
    monkeypatch.setattr(native, "files", lambda package: __import__("pathlib").Path("/missing"))
    assert "native library is missing" in native.native_error()
    assert not native.native_available()


def test_load_failure_is_explained(monkeypatch, tmp_path):
    library = tmp_path / "native" / "libmuspace_ops.so"
    library.parent.mkdir()
    library.write_bytes(b"not an ELF file")
    monkeypatch.setattr(native, "files", lambda package: tmp_path)
    assert "unable to load muSPACE-B200 native library" in native.native_error()


def test_missing_export_is_explained():
    with pytest.raises(native.NativeModuleUnavailable, match="does not export 'missing_op'"):
        native.native_function("missing_op")


def test_op_reports_unavailable_library(monkeypatch):
    from importlib import import_module

    import torch

    msda = import_module("mu_space.ops.multi_scale_deformable_attn")
    monkeypatch.setattr(native, "files", lambda package: __import__("pathlib").Path("/missing"))
    assert msda._native_extension() is None
    with pytest.raises(RuntimeError):
        msda.multi_scale_deformable_attn(
            torch.zeros(1, 4, 1, 2),
            torch.tensor([[2, 2]]),
            torch.tensor([0]),
            torch.zeros(1, 1, 1, 1, 1, 2),
            torch.ones(1, 1, 1, 1, 1),
        )


def test_tensor_descriptors_are_reused_only_for_identical_views():
    import torch

    t = torch.zeros(3, 4, 5)
    a = native._view_of(t)
    assert native._view_of(t) is a
    assert native._view_of(t.view(3, 4, 5)) is a  # another tensor object, same description
    for other in (t.transpose(0, 1), t[1:], t.view(12, 5), t.to(torch.float64), torch.zeros(3, 4, 5)):
        v = native._view_of(other)
        assert v is not a
        assert v.dl.data == (other.data_ptr() or None)
        assert v.dl.ndim == other.dim()
        assert [v.shape[i] for i in range(other.dim())] == list(other.shape)
        assert [v.strides[i] for i in range(other.dim())] == list(other.stride())

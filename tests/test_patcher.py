"""``default_patcher`` with fake mmcv / BEVFormer / UniAD modules.

Follows the MSDA cases of the reference's ``tests/test_runtime_patcher.py:13-120``,
plus the B200 compat rule: non-CUDA tensors go back to the replaced function.
"""

from __future__ import annotations

import sys
import types

import pytest
import torch

from mu_space.patcher import DefaultPatcher, PatchError
from mu_space.patcher.runtime import _MissingLegacyExtension

TARGET = "mmcv.ops.multi_scale_deform_attn"
ATTR = "multi_scale_deformable_attn_pytorch"
IMPORTED = "projects.mmdet3d_plugin.bevformer.modules.temporal_self_attention"
UNIAD_IMPORTED = "projects.mmdet3d_plugin.uniad.modules.temporal_self_attention"
EXT_LOADER = "mmcv.utils.ext_loader"


def _install_fake_module(monkeypatch, name):
    module = types.ModuleType(name)

    def original(*args, **kwargs):
        return "original"

    setattr(module, ATTR, original)
    monkeypatch.setitem(sys.modules, name, module)
    return module, original


def _install_fake_ext_loader(monkeypatch):
    module = types.ModuleType(EXT_LOADER)

    def load_ext(name, functions):
        raise ImportError(name)

    module.load_ext = load_ext
    monkeypatch.setitem(sys.modules, EXT_LOADER, module)
    return module, load_ext


def test_default_patcher_replaces_mmcv_msda_and_restores(monkeypatch):
    module, original = _install_fake_module(monkeypatch, TARGET)
    patcher = DefaultPatcher()
    report = patcher.apply()
    assert report.action == "applied"
    assert report.strict is False
    assert report.patched_modules == (TARGET,)
    assert getattr(module, ATTR) is not original
    assert getattr(module, ATTR).__name__ == "muspace_multi_scale_deformable_attn_compat"
    assert patcher.apply().action == "already-applied"
    restored = patcher.restore()
    assert restored.action == "restored"
    assert getattr(module, ATTR) is original


def test_default_patcher_updates_already_imported_bevformer_modules(monkeypatch):
    module, _ = _install_fake_module(monkeypatch, TARGET)
    imported, imported_original = _install_fake_module(monkeypatch, IMPORTED)
    report = DefaultPatcher().apply()
    assert report.patched_modules == (TARGET, IMPORTED)
    assert getattr(module, ATTR) is getattr(imported, ATTR)
    assert getattr(imported, ATTR) is not imported_original


def test_default_patcher_updates_already_imported_uniad_modules(monkeypatch):
    module, _ = _install_fake_module(monkeypatch, TARGET)
    imported, _ = _install_fake_module(monkeypatch, UNIAD_IMPORTED)
    report = DefaultPatcher().apply()
    assert report.patched_modules == (TARGET, UNIAD_IMPORTED)
    assert getattr(module, ATTR) is getattr(imported, ATTR)


def test_default_patcher_strict_mode_from_env(monkeypatch):
    module, _ = _install_fake_module(monkeypatch, TARGET)
    monkeypatch.setenv("MUSPACE_STRICT_PATCH", "1")
    report = DefaultPatcher().apply()
    assert report.strict is True
    assert getattr(module, ATTR).__name__ == "muspace_multi_scale_deformable_attn_strict"


def test_compat_wrapper_hands_cpu_tensors_back_to_the_replaced_function(monkeypatch):
    module, _ = _install_fake_module(monkeypatch, TARGET)
    patcher = DefaultPatcher()
    patcher.apply()
    value = torch.zeros(1, 4, 1, 2)
    assert getattr(module, ATTR)(value, torch.tensor([[2, 2]]), None, None) == "original"
    patcher.restore()


def test_strict_wrapper_never_falls_back(monkeypatch):
    module, _ = _install_fake_module(monkeypatch, TARGET)
    patcher = DefaultPatcher()
    patcher.apply(strict=True)
    value = torch.zeros(1, 4, 1, 2)
    loc = torch.zeros(1, 1, 1, 1, 1, 2)
    weights = torch.ones(1, 1, 1, 1, 1)
    with pytest.raises(RuntimeError, match="need CUDA tensors"):
        getattr(module, ATTR)(value, torch.tensor([[2, 2]]), loc, weights)
    patcher.restore()


def test_missing_mmcv_is_a_patch_error(monkeypatch):
    monkeypatch.setitem(sys.modules, TARGET, None)
    with pytest.raises(PatchError, match="mmcv MSDeformAttn helper is unavailable"):
        DefaultPatcher().apply()


def test_restore_releases_legacy_extension_guard(monkeypatch):
    _install_fake_module(monkeypatch, TARGET)
    ext_loader, original_load_ext = _install_fake_ext_loader(monkeypatch)
    patcher = DefaultPatcher()
    patcher.apply()
    assert ext_loader.load_ext is not original_load_ext
    assert hasattr(ext_loader, "_muspace_original_load_ext")
    patcher.restore()
    assert ext_loader.load_ext is original_load_ext
    assert not hasattr(ext_loader, "_muspace_original_load_ext")
    patcher.restore()
    assert ext_loader.load_ext is original_load_ext


def test_legacy_extension_guard_returns_placeholder_for_failed_load(monkeypatch):
    _install_fake_module(monkeypatch, TARGET)
    ext_loader, _ = _install_fake_ext_loader(monkeypatch)
    patcher = DefaultPatcher()
    patcher.apply()
    placeholder = ext_loader.load_ext("_ext", ["nms"])
    assert isinstance(placeholder, _MissingLegacyExtension)
    assert hasattr(placeholder, "nms")
    with pytest.raises(PatchError, match="mmcv._ext is unavailable"):
        placeholder.nms()
    patcher.restore()


# ---------------------------------------------------------------------------------------
# Qwen-Drive (reference tests/test_runtime_patcher.py:125-290, MSDA part)
# ---------------------------------------------------------------------------------------


def _install_fake_qwendrive(monkeypatch):
    attention = types.ModuleType("qwen_drive_perception.attention")
    ops = types.ModuleType("qwen_drive_perception.ops")

    def original_msda(*args, **kwargs):
        return ("pytorch", args, kwargs)

    def original_forward(*args, **kwargs):
        return "forward-only"

    def original_pool(*args, **kwargs):
        return "upstream-pool"

    attention.multi_scale_deformable_attn_cuda = original_msda
    ops.ms_deform_attn_bf16_forward = original_forward
    ops.voxel_pool_depth = original_pool
    for module in (attention, ops):
        monkeypatch.setitem(sys.modules, module.__name__, module)
    return attention, ops, original_msda, original_forward, original_pool


def test_qwendrive_patcher_rebinds_and_restores(monkeypatch):
    from mu_space.patcher import QwenDrivePatcher

    attention, ops, msda, forward, pool = _install_fake_qwendrive(monkeypatch)
    patcher = QwenDrivePatcher()
    first = patcher.apply()
    assert first.action == "applied" and first.strict is False
    assert attention.multi_scale_deformable_attn_cuda is not msda
    assert ops.ms_deform_attn_bf16_forward is attention.multi_scale_deformable_attn_cuda
    assert ops.voxel_pool_depth is pool  # Qwen-Drive's own CUDA code runs on CUDA GPUs
    assert patcher.apply().action == "already-applied"
    cpu = types.SimpleNamespace(dtype=torch.float32, device=types.SimpleNamespace(type="cpu"))
    assert attention.multi_scale_deformable_attn_cuda(cpu, 1, 2, 3, 4, 64)[0] == "pytorch"
    restored = patcher.restore()
    assert restored.action == "restored"
    assert attention.multi_scale_deformable_attn_cuda is msda
    assert ops.ms_deform_attn_bf16_forward is forward
    patcher.restore()
    assert attention.multi_scale_deformable_attn_cuda is msda


def test_qwendrive_msda_wrapper_routes_by_device(monkeypatch):
    from mu_space.patcher import QwenDrivePatcher

    attention, ops, *_rest = _install_fake_qwendrive(monkeypatch)
    captured = {}

    def fake_msda(*args, **kwargs):
        captured["args"], captured["kwargs"] = args, kwargs
        return "native"

    monkeypatch.setattr("muspace_b200.ops.multi_scale_deformable_attn", fake_msda)
    patcher = QwenDrivePatcher()
    patcher.apply()
    wrapper = attention.multi_scale_deformable_attn_cuda
    cuda = types.SimpleNamespace(dtype=torch.bfloat16, device=types.SimpleNamespace(type="cuda"))
    assert wrapper(cuda, "shapes", "starts", "locations", "weights", im2col_step=64) == "native"
    assert captured["kwargs"] == {"im2col_step": 64, "backend": "auto"}
    assert captured["args"][1:] == ("shapes", "starts", "locations", "weights")
    with pytest.raises(TypeError, match="bfloat16"):
        wrapper(types.SimpleNamespace(dtype=torch.float32, device=types.SimpleNamespace(type="cuda")),
                None, None, None, None, 64)
    cpu = types.SimpleNamespace(dtype=torch.float32, device=types.SimpleNamespace(type="cpu"))
    assert wrapper(cpu, "shapes", "starts", "locations", "weights", 64)[0] == "pytorch"
    assert ops.ms_deform_attn_bf16_forward is wrapper
    patcher.restore()
    patcher.apply(strict=True)
    attention.multi_scale_deformable_attn_cuda(cuda, "s", "t", "l", "w", 32)
    assert captured["kwargs"] == {"im2col_step": 32, "backend": "cuda"}
    patcher.restore()


def test_qwendrive_patcher_rejects_a_partial_package(monkeypatch):
    from mu_space.patcher import QwenDrivePatcher

    attention, ops, *_rest = _install_fake_qwendrive(monkeypatch)
    del ops.ms_deform_attn_bf16_forward
    with pytest.raises(PatchError, match="ms_deform_attn_bf16_forward"):
        QwenDrivePatcher().apply()
    assert attention.multi_scale_deformable_attn_cuda(None)[0] == "pytorch"


def test_qwendrive_patcher_without_the_package_is_a_patch_error(monkeypatch):
    from mu_space.patcher import QwenDrivePatcher

    monkeypatch.setitem(sys.modules, "qwen_drive_perception", None)
    monkeypatch.delitem(sys.modules, "qwen_drive_perception.attention", raising=False)
    with pytest.raises(PatchError, match="PYTHONPATH"):
        QwenDrivePatcher().apply()


@pytest.mark.gpu
def test_qwendrive_wrapper_runs_forward_and_backward_on_the_b200_kernels(monkeypatch, cuda_device):
    """Qwen-Drive's kernel is forward-only; through the wrapper its bf16 MSDA
    gets gradients, equal to the fp32 oracle on the same quantised inputs."""
    from mu_space.patcher import QwenDrivePatcher
    from muspace_b200 import cases
    from oracle import oracle_backward, oracle_forward

    attention, *_rest = _install_fake_qwendrive(monkeypatch)
    patcher = QwenDrivePatcher()
    patcher.apply()
    try:
        cfg = cases.CONFIGS["c2"].with_(batch=1, queries=64)
        inp = cases.make_inputs(cfg, dtype=torch.bfloat16, device=cuda_device)
        names = ("value", "spatial_shapes", "level_start_index", "sampling_locations", "attention_weights")
        leaves = {k: (inp[k].clone().requires_grad_(True) if inp[k].is_floating_point() else inp[k]) for k in names}
        out = attention.multi_scale_deformable_attn_cuda(*[leaves[k] for k in names], 64)
        out.backward(inp["grad_output"])
        host = [inp[k].float().cpu().numpy() if inp[k].is_floating_point() else inp[k].cpu().numpy() for k in names]
        exp_out = oracle_forward(*host)
        _, exp_gl, exp_gw = oracle_backward(*host, inp["grad_output"].float().cpu().numpy())
        torch.testing.assert_close(out.float().cpu(), torch.from_numpy(exp_out), rtol=2e-2, atol=2e-2)
        torch.testing.assert_close(leaves["sampling_locations"].grad.float().cpu(), torch.from_numpy(exp_gl),
                                   rtol=2e-2, atol=2e-2)
        torch.testing.assert_close(leaves["attention_weights"].grad.float().cpu(), torch.from_numpy(exp_gw),
                                   rtol=2e-2, atol=2e-2)
    finally:
        patcher.restore()

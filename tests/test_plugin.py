"""The plug-in installer (heimdall_b200.plugin) on stand-in modules: what it patches, that it restores the
originals, and that it refuses CPU devices and CPU tensors (there is no CPU path).  No GPU needed.

The stand-ins carry the attribute names of the reference modules around the Bifrost path
(heimdall/kernels.py:132-155, heimdall/hibrit.py:32 and the HybridAttention methods, heimdall/motor.py:70);
the installer replaces the HybridAttention methods and motor.delta_rule_gqa and leaves the rest."""
import types

import pytest
import torch


def fake_modules():
    def orig(*a, **k):
        raise AssertionError("original called")

    kernels = types.ModuleType("heimdall.kernels")
    kernels.delta_rule = kernels.delta_rule_step = orig
    kernels.delta_rule_reference = orig
    hibrit = types.ModuleType("heimdall.hibrit")
    hibrit.delta_rule = hibrit.delta_rule_step = orig

    class HybridAttention(torch.nn.Module):
        _student = _window = _mem_inputs = _teacher = orig
    hibrit.HybridAttention = HybridAttention
    motor = types.ModuleType("heimdall.motor")
    motor.delta_rule_gqa = motor.window_attention = orig
    return {"kernels": kernels, "hibrit": hibrit, "motor": motor}, orig


def test_install_patches_and_uninstall_restores():
    from heimdall_b200 import plugin
    m, orig = fake_modules()
    plugin.install(m)
    try:
        assert plugin.installed()
        # the linear-attention ops stay the reference's (other layers of the model call them)
        assert m["kernels"].delta_rule is orig and m["kernels"].delta_rule_step is orig
        assert m["hibrit"].delta_rule is orig and m["hibrit"].delta_rule_step is orig
        assert m["motor"].delta_rule_gqa is plugin.delta_rule_gqa
        assert m["motor"].window_attention is plugin.window_attention
        cls = m["hibrit"].HybridAttention
        assert cls._student is plugin._student and cls._window is plugin._window
        assert cls._mem_inputs is plugin._mem_inputs and cls._teacher is plugin._teacher
        plugin.install(m)            # idempotent
    finally:
        plugin.uninstall()
    assert not plugin.installed()
    assert m["kernels"].delta_rule is orig and m["motor"].delta_rule_gqa is orig
    assert m["hibrit"].HybridAttention._student is orig


def test_install_is_all_or_nothing():
    from heimdall_b200 import plugin
    m, orig = fake_modules()
    del m["motor"].delta_rule_gqa
    with pytest.raises(AttributeError):
        plugin.install(m)
    assert not plugin.installed() and m["kernels"].delta_rule is orig


def test_patched_ops_refuse_cpu_tensors_and_prepare_refuses_cpu():
    from heimdall_b200 import plugin
    m, _ = fake_modules()
    with pytest.raises(RuntimeError, match="CUDA"):
        plugin.prepare(torch.device("cpu"), modules=m)
    assert not plugin.installed()
    z = torch.zeros(1, 4, 1, 256)
    with pytest.raises(RuntimeError, match="CUDA"):
        plugin.delta_rule(z, z, z, z[..., 0], z[..., 0])
    with pytest.raises(RuntimeError, match="CUDA"):
        plugin.delta_rule_step(z[:, 0], z[:, 0], z[:, 0], z[:, 0, :, 0], z[:, 0, :, 0], torch.zeros(1, 1, 256, 256))

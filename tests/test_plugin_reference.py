"""The plug-in installed into the real reference package (no GPU needed).

Runs only when the reference project is available: set HEIMDALL_REFERENCE to its directory (the one that
holds the ``heimdall`` package, or its parent).  Checks that ``plugin.install()`` replaces exactly the
Bifrost-path names and leaves the model's other callers of the delta rule on the reference's own ops: the
Qwen3.5 linear-attention layers (``GatedDeltaNet.forward``, heimdall/hibrit.py:159-185) call the module-level
``delta_rule`` / ``delta_rule_step`` with their own head sizes, which the head-dim-256 kernels do not cover.
"""
import sys

import pytest
import torch

from conftest import reference_project
from params import module_config


@pytest.fixture()
def heimdall_modules():
    ref = reference_project()
    if ref is None:
        pytest.skip("reference not available (set HEIMDALL_REFERENCE to the reference project)")
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    import heimdall.hibrit as hb
    import heimdall.kernels as hk
    import heimdall.motor as hm
    return {"kernels": hk, "hibrit": hb, "motor": hm}


def _names(m):
    hb = m["hibrit"]
    A = hb.HybridAttention
    return {("kernels", "delta_rule"): m["kernels"].delta_rule,
            ("kernels", "delta_rule_step"): m["kernels"].delta_rule_step,
            ("hibrit", "delta_rule"): hb.delta_rule, ("hibrit", "delta_rule_step"): hb.delta_rule_step,
            ("motor", "delta_rule_gqa"): m["motor"].delta_rule_gqa,
            ("motor", "window_attention"): m["motor"].window_attention,
            ("hibrit", "HybridAttention._student"): A.__dict__["_student"],
            ("hibrit", "HybridAttention._mem_inputs"): A.__dict__["_mem_inputs"],
            ("hibrit", "HybridAttention._window"): A.__dict__["_window"],
            ("hibrit", "HybridAttention._teacher"): A.__dict__["_teacher"]}


def test_install_replaces_only_the_bifrost_path(heimdall_modules):
    from heimdall_b200 import plugin
    m = heimdall_modules
    before = _names(m)
    hb = m["hibrit"]
    # a Qwen3.5 linear-attention layer (head dim 16) on CPU, before the install
    c = hb.HybridConfig(module_config(4, 2, 32, 64))
    torch.manual_seed(0)
    lin = hb.GatedDeltaNet(c).eval()
    x = torch.randn(1, 40, 64)
    with torch.no_grad():
        y0 = lin(x, {}, 0)
    plugin.install()
    try:
        after = _names(m)
        changed = {k for k in before if after[k] is not before[k]}
        assert changed == set(plugin.PATCHED_NAMES)
        # the linear-attention layer still runs the reference's ops (prefill, then one cached decode token)
        cache = {}
        with torch.no_grad():
            y1 = lin(x, cache, 0)
            lin(torch.randn(1, 1, 64), cache, 40)
        assert torch.equal(y0, y1)
        # the Bifrost layer core is the B200 one: it refuses CPU tensors instead of falling back
        a = hb.HybridAttention(hb.HybridConfig(module_config(4, 2, 32, 64)))
        a.convert(8, 2, 1, "long")
        t = torch.zeros(1, 3, 4, 32)
        with pytest.raises(RuntimeError, match="CUDA"):
            a._student(torch.zeros(1, 3, 64), t, t[:, :, :2], t[:, :, :2], t.transpose(1, 2),
                       t[:, :, :2].transpose(1, 2), 0, None)
    finally:
        plugin.uninstall()
    assert all(_names(m)[k] is v for k, v in before.items())

"""The plug-in installed into stand-in reference modules on a GPU: prepare() self-tests against the host's
delta_rule_reference (here the oracle's restatement of it), then every patched entry point answers like the
oracle.  The stand-in HybridAttention carries the converted parameters under the reference's attribute names
(heimdall/hibrit.py:211-240)."""
import pytest
import torch

from oracle import bifrost_oracle as ob
from params import layer_params
from test_plugin import fake_modules

pytestmark = pytest.mark.gpu
O_TOL = 2e-3


def _attn(p, H, G, D, d, dev):
    a = torch.nn.Module()
    a.fq, a.fk = torch.nn.Parameter(p.fq.clone()), torch.nn.Parameter(p.fk.clone())
    a.ab, a.mix = torch.nn.Linear(d, 2 * G), torch.nn.Linear(d, H)
    with torch.no_grad():
        a.ab.weight.copy_(p.ab_w), a.ab.bias.copy_(p.ab_b), a.mix.weight.copy_(p.mix_w), a.mix.bias.copy_(p.mix_b)
    for n in ("mix_lse", "mem_scale", "A_log", "dt_bias"):
        setattr(a, n, torch.nn.Parameter(getattr(p, n).clone()))
    a.register_buffer("decay_mask", p.decay_mask.clone())
    a.window, a.sinks = p.window, p.sinks
    return a.to(dev)


def test_prepare_installs_and_routes_every_entry_point():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda")
    from heimdall_b200 import plugin
    m, _ = fake_modules()
    m["kernels"].delta_rule_reference = lambda q, k, v, g, beta, chunk, s0: ob.gdn_chunked(q, k, v, g, beta, chunk, s0)
    desc = plugin.prepare(dev, modules=m)
    try:
        assert desc.startswith("heimdall_b200") and plugin.installed()
        H, G, D, d, W, S, T = 24, 4, 256, 128, 128, 4, 300
        p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=3)
        cls = m["hibrit"].HybridAttention
        attn = _attn(p, H, G, D, d, dev)
        gen = torch.Generator().manual_seed(8)
        rms = lambda z: z * torch.rsqrt(z.square().mean(-1, keepdim=True) + 1e-6)
        bf = lambda z: z.to(torch.bfloat16)
        x = bf(torch.randn(1, T, d, generator=gen))
        q, k, v = (bf(rms(torch.randn(1, T, n, D, generator=gen))) for n in (H, G, G))
        qr, kr = bf(rms(torch.randn(1, H, T, D, generator=gen))), bf(rms(torch.randn(1, G, T, D, generator=gen)))
        f, cu = (lambda z: z.float()), (lambda z: z.to(dev))
        # _student: prefill with a cache, then one decode step
        cache, cache_r = {}, {}
        o = cls._student(attn, cu(x[:, :-1]), cu(q[:, :-1]), cu(k[:, :-1]), cu(v[:, :-1]), cu(qr[:, :, :-1]),
                         cu(kr[:, :, :-1]), 0, cache)
        o_r = ob.student(p, f(x[:, :-1]), f(q[:, :-1]), f(k[:, :-1]), f(v[:, :-1]), f(qr[:, :, :-1]),
                         f(kr[:, :, :-1]), 0, cache_r)
        assert ob.rel_l2(o.cpu(), o_r) < O_TOL
        o = cls._student(attn, cu(x[:, -1:]), cu(q[:, -1:]), cu(k[:, -1:]), cu(v[:, -1:]), cu(qr[:, :, -1:]),
                         cu(kr[:, :, -1:]), T - 1, cache)
        o_r = ob.student(p, f(x[:, -1:]), f(q[:, -1:]), f(k[:, -1:]), f(v[:, -1:]), f(qr[:, :, -1:]),
                         f(kr[:, :, -1:]), T - 1, cache_r)
        assert ob.rel_l2(o.cpu(), o_r) < O_TOL
        # _mem_inputs with explicit positions
        pos = torch.arange(T)
        got = cls._mem_inputs(attn, cu(x), cu(q), cu(k), cu(pos))
        ref = ob.mem_inputs(p, f(x), f(q), f(k), pos)
        for a_, b_ in zip(got, ref):
            assert ob.rel_l2(a_.cpu(), b_) < 1e-3
        # _window with the reference's empty-ring layout (motor.window_attention, heimdall/motor.py:105-115)
        vt = v.transpose(1, 2)
        ext_pos = torch.cat((torch.full((W,), -1, dtype=torch.long), pos))
        ext_k = torch.cat((kr.new_zeros(1, G, W, D), kr), 2)
        ext_v = torch.cat((vt.new_zeros(1, G, W, D), vt), 2)
        o, lse = cls._window(attn, cu(qr), cu(ext_k), cu(ext_v), cu(ext_pos), cu(kr[:, :, :S]), cu(vt[:, :, :S]),
                             cu(pos))
        o_r, lse_r = ob.window_attention(f(qr), f(ext_k), f(ext_v), ext_pos, f(kr[:, :, :S]), f(vt[:, :, :S]), pos,
                                         W, S)
        assert ob.rel_l2(o.cpu(), o_r) < O_TOL and (lse.cpu() - lse_r).abs().max() < 1e-3
        # motor.window_attention itself (patched: the sequence's own keys from position 0, no host read)
        o2, lse2 = m["motor"].window_attention(attn, cu(qr), cu(kr), cu(v))
        assert ob.rel_l2(o2.cpu(), o_r) < O_TOL and (lse2.cpu() - lse_r).abs().max() < 1e-3
        # _window at a later start (ring of earlier positions, then the new tokens)
        st = 1000
        pos2 = torch.arange(st, st + T)
        ext_pos2 = torch.cat((torch.arange(st - W, st), pos2))
        ext_k2 = torch.cat((bf(rms(torch.randn(1, G, W, D, generator=gen))), kr), 2)
        ext_v2 = torch.cat((bf(rms(torch.randn(1, G, W, D, generator=gen))), vt), 2)
        o, lse = cls._window(attn, cu(qr), cu(ext_k2), cu(ext_v2), cu(ext_pos2), cu(kr[:, :, :S]), cu(vt[:, :, :S]),
                             cu(pos2))
        o_r, lse_r = ob.window_attention(f(qr), f(ext_k2), f(ext_v2), ext_pos2, f(kr[:, :, :S]), f(vt[:, :, :S]),
                                         pos2, W, S)
        assert ob.rel_l2(o.cpu(), o_r) < O_TOL and (lse.cpu() - lse_r).abs().max() < 1e-3
        bad = ext_pos.clone()
        bad[W + 5] = -1               # a hole inside the window: not the contiguous form
        with pytest.raises(NotImplementedError):
            cls._window(attn, cu(qr), cu(ext_k), cu(ext_v), cu(bad), cu(kr[:, :, :S]), cu(vt[:, :, :S]), cu(pos))
        # the B200 op by name (exported by the plugin; the module-level op of the host package is left to
        # its linear-attention layers)
        assert m["kernels"].delta_rule is not plugin.delta_rule
        g = -torch.rand(1, T, G, generator=gen) * 0.1
        beta = torch.rand(1, T, G, generator=gen)
        kn = torch.nn.functional.normalize(f(k), dim=-1)
        o, s = plugin.delta_rule(cu(kn), cu(kn), cu(f(v)), cu(g), cu(beta), 64, None)
        o_r, s_r = ob.gdn_chunked(kn, kn, f(v), g, beta, 64, None)
        assert ob.rel_l2(o.cpu(), o_r) < O_TOL and ob.rel_l2(s.cpu(), s_r) < 1e-3
        # parameters updated in place -> the cached layer is rebuilt
        with torch.no_grad():
            attn.mem_scale.mul_(0.5)
        assert plugin.layer_for(attn, dev).p["mem_scale"].allclose(attn.mem_scale)
    finally:
        plugin.uninstall()

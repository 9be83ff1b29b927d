"""Pin the CPU oracle against the reference's own outputs (golden fixtures) and its own test pins.

The fixtures were written by ``tests/golden/make_golden.py``, which runs Heimdall's
``delta_rule_reference`` / ``delta_rule_step`` / ``delta_rule_gqa`` / ``HybridAttention._student``
unmodified.  These tests run on the CPU only.
"""
import pytest
import torch

from oracle import bifrost_oracle as ob
from params import layer_params


def _close(a, b, tol):
    return (a.double() - b.double()).abs().max().item() <= tol * max(1.0, b.abs().max().item())


@pytest.mark.parametrize("case", ["gdn_small", "gdn_prepare", "gdn_d256"])
def test_gdn_chunked_matches_reference(golden_gdn, case):
    c = golden_gdn[case]
    o, S = ob.gdn_chunked(c["q"], c["k"], c["v"], c["g"], c["beta"], c["chunk"], c["s0"])
    assert _close(o, c["o"], 1e-5) and _close(S, c["S"], 1e-5)
    assert ob.rel_l2(o, c["o"]) < 1e-6 and ob.rel_l2(S, c["S"]) < 1e-6


def test_gdn_chunk_equals_recurrence(golden_gdn):
    """Reference pin tests/test_heimdall.py:36-48: chunked == token loop, atol 1e-4."""
    c = golden_gdn["gdn_small"]
    o, S = ob.gdn_recurrent(c["q"], c["k"], c["v"], c["g"], c["beta"], c["s0"])
    assert torch.allclose(o, c["o_rec"], atol=1e-5) and torch.allclose(S, c["S_rec"], atol=1e-5)
    assert torch.allclose(o, c["o"], atol=1e-4) and torch.allclose(S, c["S"], atol=1e-4)


def test_gdn_step_matches_reference(golden_gdn):
    c = golden_gdn["gdn_step"]
    o, S = ob.gdn_step(c["q"], c["k"], c["v"], c["g"], c["beta"], c["s0"])
    assert _close(o, c["o"], 1e-6) and _close(S, c["S"], 1e-6)


def test_gdn_gqa_matches_reference(golden_gdn):
    """Reference pin tests/test_motor.py:28-39 shapes (G=2, R=3, D=8, chunk 16)."""
    c = golden_gdn["gdn_gqa"]
    o, S = ob.gdn_gqa(c["q"], c["k"], c["v"], c["g"], c["beta"], c["chunk"], c["s0"])
    assert (o - c["o"]).abs().max() < 1e-5 and (S - c["S"]).abs().max() < 1e-5


def test_gdn_gqa_equals_repeated_heads(golden_gdn):
    c = golden_gdn["gdn_gqa"]
    B, T, G, R, D = c["q"].shape
    rep = lambda z: z.repeat_interleave(R, 2)
    o_ref, s_ref = ob.gdn_chunked(c["q"].reshape(B, T, G * R, D), rep(c["k"]), rep(c["v"]), rep(c["g"]),
                                  rep(c["beta"]), 16, c["s0"].repeat_interleave(R, 1))
    o, s = ob.gdn_gqa(c["q"], c["k"], c["v"], c["g"], c["beta"], 16, c["s0"])
    assert (o.reshape(B, T, G * R, D) - o_ref).abs().max() < 1e-5 and (s - s_ref[:, ::R]).abs().max() < 1e-5


def test_chunk_size_invariance(golden_gdn):
    """The chunk size is an implementation choice: 16/32/64/128 agree with the recurrent form."""
    c = golden_gdn["gdn_d256"]
    o_rec, s_rec = ob.gdn_recurrent(c["q"], c["k"], c["v"], c["g"], c["beta"], c["s0"], dtype=torch.float64)
    for C in (16, 32, 64, 128):
        o, s = ob.gdn_chunked(c["q"], c["k"], c["v"], c["g"], c["beta"], C, c["s0"])
        assert ob.rel_l2(o, o_rec) < 1e-5 and ob.rel_l2(s, s_rec) < 1e-5


def _layer(golden_layer, name):
    c = golden_layer[name]
    p = layer_params(c["H"], c["G"], c["D"], c["d"], c["window"], c["sinks"], c["archival"], c["seed"])
    return c, p


@pytest.mark.parametrize("name", ["tiny", "d256"])
def test_params_regenerate(golden_layer, name):
    c, p = _layer(golden_layer, name)
    got = dict(fq=p.fq, fk=p.fk, **{"ab.weight": p.ab_w, "ab.bias": p.ab_b, "mix.weight": p.mix_w,
                                     "mix.bias": p.mix_b}, mix_lse=p.mix_lse, mem_scale=p.mem_scale,
               A_log=p.A_log, dt_bias=p.dt_bias)
    for k, s in c["param_sums"].items():
        assert abs(float(got[k].double().sum()) - s) <= 1e-6 * max(1.0, abs(s)), k


def test_window_matches_reference(golden_layer):
    c, p = _layer(golden_layer, "tiny")
    T, W, S, D, G = c["q"].shape[1], c["window"], c["sinks"], c["D"], c["G"]
    kr, vt = c["kr"].float(), c["v"].float().transpose(1, 2)
    ext_k = torch.cat((kr.new_zeros(1, G, W, D), kr), 2)
    ext_v = torch.cat((vt.new_zeros(1, G, W, D), vt), 2)
    ext_pos = torch.cat((torch.full((W,), -1, dtype=torch.long), torch.arange(T)))
    o, lse = ob.window_attention(c["qr"].float(), ext_k, ext_v, ext_pos, kr[:, :, :S], vt[:, :, :S],
                                 torch.arange(T), W, S)
    assert _close(o, c["o_win"], 1e-5) and _close(lse, c["lse"], 1e-5)


@pytest.mark.parametrize("name", ["tiny", "d256"])
def test_student_matches_reference(golden_layer, name):
    """Mixed prefill/decode parts (reference pin tests/test_hibrit.py:78-90) through the cache dict."""
    c, p = _layer(golden_layer, name)
    f = lambda k: c[k].float()
    cache, outs, s = {}, [], 0
    for n in c["parts"]:
        sl = slice(s, s + n)
        outs.append(ob.student(p, f("x")[:, sl], f("q")[:, sl], f("k")[:, sl], f("v")[:, sl],
                               f("qr")[:, :, sl], f("kr")[:, :, sl], s, cache))
        s += n
    o = torch.cat(outs, 1)
    assert _close(o, c["o_parts"], 2e-5), (o - c["o_parts"]).abs().max()
    for k, ref in c["cache"].items():
        got = cache[k]
        assert got.shape == ref.shape, k
        assert _close(got.double(), ref.double(), 2e-5), k
    # and the whole sequence in one call equals the parts (reference: full == chunked within 1e-4)
    full = ob.student(p, f("x"), f("q"), f("k"), f("v"), f("qr"), f("kr"), 0, None)
    assert (full - o).abs().max() < 1e-4
    assert c["full_vs_parts"] < 1e-4


def test_window_only_mode_ignores_memory(golden_layer):
    """memory=False is the reference's "window" mode: before W the outputs agree with memory on."""
    c, p = _layer(golden_layer, "tiny")
    f = lambda k: c[k].float()
    a = ob.student(p, f("x"), f("q"), f("k"), f("v"), f("qr"), f("kr"), 0, None, memory=True)
    b = ob.student(p, f("x"), f("q"), f("k"), f("v"), f("qr"), f("kr"), 0, None, memory=False)
    W = c["window"]
    assert (a[:, :W] - b[:, :W]).abs().max() < 1e-6
    assert (a[:, W:] - b[:, W:]).abs().max() > 1e-4


def test_oracle_against_live_reference():
    """When the reference project is available (HEIMDALL_REFERENCE), compare the oracle to it on fresh seeds."""
    import sys
    from conftest import reference_project
    ref = reference_project()
    if ref is None:
        pytest.skip("reference not available (set HEIMDALL_REFERENCE to the reference project)")
    sys.path.insert(0, str(ref))
    import torch.nn.functional as F
    from heimdall.kernels import delta_rule_reference
    from heimdall.motor import delta_rule_gqa
    torch.manual_seed(123)
    B, T, G, R, D = 2, 131, 2, 3, 32
    q = torch.randn(B, T, G, R, D)
    k = F.normalize(torch.randn(B, T, G, D), dim=-1)
    v, g, beta = torch.randn(B, T, G, D), -torch.rand(B, T, G), torch.rand(B, T, G)
    s0 = torch.randn(B, G, D, D) * 0.1
    o1, s1 = delta_rule_gqa(q, k, v, g, beta, 64, s0)
    o2, s2 = ob.gdn_gqa(q, k, v, g, beta, 64, s0)
    assert (o1 - o2).abs().max() < 1e-5 and (s1 - s2).abs().max() < 1e-5
    o3, s3 = delta_rule_reference(q[:, :, :, 0], k, v, g, beta, 32, s0)
    o4, s4 = ob.gdn_chunked(q[:, :, :, 0], k, v, g, beta, 32, s0)
    assert (o3 - o4).abs().max() < 1e-5 and (s3 - s4).abs().max() < 1e-5


def test_student_reference_form_equals_gqa_form(golden_layer):
    """The oracle's statement-for-statement form of the reference's prefill memory (state repeated per query
    head, hibrit.py:404-408) equals its GQA-native form (the reference's pin tests/test_motor.py:28-39), and
    both match the reference's own outputs."""
    c, p = _layer(golden_layer, "d256")
    f = lambda k: c[k].float()
    a = ob.student(p, f("x"), f("q"), f("k"), f("v"), f("qr"), f("kr"), 0, None)
    b = ob.student(p, f("x"), f("q"), f("k"), f("v"), f("qr"), f("kr"), 0, None, gqa_native=False)
    assert (a - b).abs().max() < 1e-5


@pytest.mark.parametrize("name", ["d256", "d256_window"])
def test_attention_forward_matches_reference(golden_forward, name):
    """The whole converted attention layer (projections, ZNorm, partial RoPE, the core, output gate and o_proj;
    HybridAttention.forward, hibrit.py:426-432) over mixed prefill/decode parts, against the reference."""
    from params import proj_params
    c = golden_forward[name]
    p = layer_params(c["H"], c["G"], c["D"], c["d"], c["window"], c["sinks"], c["archival"], c["seed"])
    pp = proj_params(c["H"], c["G"], c["D"], c["d"], c["seed"], c["rot"], c["theta"])
    cache, outs, s = {}, [], 0
    for n in c["parts"]:
        outs.append(ob.attention_forward(p, pp, c["x"][:, s:s + n], cache, s, memory=c["mode"] != "window"))
        s += n
    y = torch.cat(outs, 1)
    assert _close(y, c["y_parts"], 2e-5), (y - c["y_parts"]).abs().max()
    for k, ref in c["cache"].items():
        assert _close(cache[k].double(), ref.double(), 2e-5), k

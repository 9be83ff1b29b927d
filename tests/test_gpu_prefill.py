"""GPU parity: chunked delta rule (tcgen05), window + sink attention (tcgen05), fused layer prefill.

CUDA results are compared with the reference's own outputs (golden fixtures) and with the CPU oracle on
seeded bf16-valued inputs.  Tolerances (north star): outputs rel-L2 <= 2e-3, states rel-L2 <= 1e-3.
"""
import math

import pytest
import torch
import torch.nn.functional as F

from oracle import bifrost_oracle as ob
from params import layer_params

pytestmark = pytest.mark.gpu

O_TOL, S_TOL = 2e-3, 1e-3


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


def _gdn_inputs(B, T, G, R, D, seed, s0_scale=0.05, archival=False):
    gen = torch.Generator().manual_seed(seed)
    q = F.normalize(torch.randn(B, T, G, R, D, generator=gen), dim=-1) * D ** -0.5
    k = F.normalize(torch.randn(B, T, G, D, generator=gen), dim=-1)
    v = torch.randn(B, T, G, D, generator=gen)
    beta = torch.sigmoid(torch.randn(B, T, G, generator=gen))
    A_log = torch.empty(G).uniform_(-4, 0, generator=gen)
    g = -A_log.exp() * F.softplus(torch.randn(B, T, G, generator=gen))
    if archival:
        g[..., 0] = 0.0
    s0 = None if s0_scale == 0 else torch.randn(B, G, D, D, generator=gen) * s0_scale
    return q, k, v, g, beta, s0


def test_delta_rule_golden_d256(golden_gdn):
    """The reference's delta_rule_reference output at D=256, ragged T=70, with an initial state."""
    dev = _dev()
    import heimdall_b200 as hb
    c = golden_gdn["gdn_d256"]
    o, S = hb.delta_rule(*(z.to(dev) for z in (c["q"], c["k"], c["v"], c["g"], c["beta"])), 64, c["s0"].to(dev))
    torch.cuda.synchronize()
    assert ob.rel_l2(o.cpu(), c["o"]) < O_TOL and ob.rel_l2(S.cpu(), c["S"]) < S_TOL


@pytest.mark.parametrize("T", [1, 127, 128, 129, 300])
def test_delta_rule_gqa_vs_oracle(T):
    dev = _dev()
    import heimdall_b200 as hb
    B, G, R, D = 2, 4, 6, 256
    q, k, v, g, beta, s0 = _gdn_inputs(B, T, G, R, D, seed=T)
    o_ref, s_ref = ob.gdn_gqa(q, k, v, g, beta, 64, s0, dtype=torch.float64)
    o, s = hb.delta_rule_gqa(*(z.to(dev) for z in (q, k, v, g, beta)), 64, s0.to(dev))
    torch.cuda.synchronize()
    assert ob.rel_l2(o.cpu(), o_ref) < O_TOL and ob.rel_l2(s.cpu(), s_ref) < S_TOL


def test_delta_rule_config0_full_size():
    """BASELINE config 0 at full size: B=1, H=4, T=4096, D=256, fp32, zero initial state, one archival head;
    compared with the recurrent form (the reference's own check), in float64."""
    dev = _dev()
    import heimdall_b200 as hb
    B, H, T, D = 1, 4, 4096, 256
    q, k, v, g, beta, _ = _gdn_inputs(B, T, H, 1, D, seed=0, s0_scale=0, archival=True)
    q = q[:, :, :, 0] * D ** 0.5   # config 0: q is unit-norm (no extra scale)
    o_ref, s_ref = ob.gdn_chunked(q, k, v, g, beta, 64, None, dtype=torch.float64)
    o, s = hb.delta_rule(*(z.to(dev) for z in (q, k, v, g, beta)))
    torch.cuda.synchronize()
    eo, es = ob.rel_l2(o.cpu(), o_ref), ob.rel_l2(s.cpu(), s_ref)
    assert eo < O_TOL and es < S_TOL, (eo, es)


def _bf(*ts):
    return [t.to(torch.bfloat16) for t in ts]


@pytest.mark.parametrize("T,W,start", [(600, 256, 0), (333, 200, 0), (300, 128, 700), (5, 16, 0)])
def test_window_vs_oracle(T, W, start):
    dev = _dev()
    import heimdall_b200 as hb
    B, H, G, D, S = 2, 24, 4, 256, 4
    gen = torch.Generator().manual_seed(T + W)
    rms = lambda z: z * torch.rsqrt(z.square().mean(-1, keepdim=True) + 1e-6)
    nring = W if start > 0 else 0
    Tk = nring + T
    qr, = _bf(rms(torch.randn(B, H, T, D, generator=gen)))
    ek, ev = _bf(rms(torch.randn(B, G, Tk, D, generator=gen)), rms(torch.randn(B, G, Tk, D, generator=gen)))
    sk, sv = _bf(rms(torch.randn(B, G, S, D, generator=gen)), rms(torch.randn(B, G, S, D, generator=gen)))
    pos = torch.arange(start, start + T)
    kpos0 = start - nring
    ext_pos = torch.arange(kpos0, kpos0 + Tk)
    if start == 0:
        # sinks are the first S tokens themselves
        sk, sv = ek[:, :, :S], ev[:, :, :S]
    # oracle: the reference's ext layout is [ring W rows; new tokens]; without history the ring rows are empty
    ok_, ov_, op_ = ek.float(), ev.float(), ext_pos
    if nring == 0:
        ok_ = torch.cat((ok_.new_zeros(B, G, W, D), ok_), 2)
        ov_ = torch.cat((ov_.new_zeros(B, G, W, D), ov_), 2)
        op_ = torch.cat((torch.full((W,), -1, dtype=torch.long), op_))
    o_ref, lse_ref = ob.window_attention(qr.float(), ok_, ov_, op_, sk.float(), sv.float(), pos, W, S,
                                         dtype=torch.float64)
    o, lse = hb.window_attention(qr.to(dev), ek.to(dev), ev.to(dev), start, kpos0, S, W, sk.to(dev), sv.to(dev))
    torch.cuda.synchronize()
    assert ob.rel_l2(o.cpu(), o_ref) < O_TOL
    assert (lse.cpu().double() - lse_ref).abs().max() < 1e-3


def _layer_inputs(H, G, D, d, T, seed, B=1):
    gen = torch.Generator().manual_seed(seed)
    rms = lambda z: z * torch.rsqrt(z.square().mean(-1, keepdim=True) + 1e-6)
    bf = lambda z: z.to(torch.bfloat16)
    x = bf(torch.randn(B, T, d, generator=gen))
    q = bf(rms(torch.randn(B, T, H, D, generator=gen)))
    k = bf(rms(torch.randn(B, T, G, D, generator=gen)))
    v = bf(rms(torch.randn(B, T, G, D, generator=gen)))
    qr = bf(rms(torch.randn(B, H, T, D, generator=gen)))
    kr = bf(rms(torch.randn(B, G, T, D, generator=gen)))
    return x, q, k, v, qr, kr


def test_layer_golden_mixed_parts(golden_layer):
    """Reference HybridAttention._student outputs over mixed prefill/decode parts (10,1,13,1,5), D=256."""
    dev = _dev()
    from heimdall_b200 import BifrostLayer
    c = golden_layer["d256"]
    p = layer_params(c["H"], c["G"], c["D"], c["d"], c["window"], c["sinks"], c["archival"], c["seed"])
    L = BifrostLayer.from_params(p, dev)
    cache, outs, s = {}, [], 0
    for n in c["parts"]:
        sl = slice(s, s + n)
        outs.append(L.student(c["x"][:, sl].to(dev), c["q"][:, sl].to(dev), c["k"][:, sl].to(dev),
                              c["v"][:, sl].to(dev), c["qr"][:, :, sl].to(dev), c["kr"][:, :, sl].to(dev), s, cache))
        s += n
    o = torch.cat(outs, 1).cpu()
    assert ob.rel_l2(o, c["o_parts"]) < O_TOL
    assert ob.rel_l2(cache["S"].cpu(), c["cache"]["S"]) < S_TOL
    assert torch.equal(cache["ring_pos"].cpu(), c["cache"]["ring_pos"])
    assert ob.rel_l2(cache["ring_km"].cpu(), c["cache"]["ring_km"]) < 1e-3
    assert torch.equal(cache["sink_k"].cpu().float(), c["cache"]["sink_k"].float())


@pytest.mark.parametrize("T,W,memory", [(1000, 256, True), (700, 200, True), (400, 256, False), (100, 256, True)])
def test_layer_prefill_vs_oracle(T, W, memory):
    dev = _dev()
    from heimdall_b200 import BifrostLayer
    H, G, D, d, S = 24, 4, 256, 128, 4
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=W)
    x, q, k, v, qr, kr = _layer_inputs(H, G, D, d, T, seed=T)
    f = lambda z: z.float()
    o_ref = ob.student(p, f(x), f(q), f(k), f(v), f(qr), f(kr), 0, None, memory=memory, dtype=torch.float64)
    L = BifrostLayer.from_params(p, dev)
    o = L.student(x.to(dev), q.to(dev), k.to(dev), v.to(dev), qr.to(dev), kr.to(dev), 0, None, memory=memory)
    torch.cuda.synchronize()
    assert ob.rel_l2(o.cpu(), o_ref) < O_TOL


@pytest.mark.parametrize("parts,W", [((300, 1, 257, 1, 1, 440), 256), ((129, 72, 1, 200), 200)])
def test_layer_mixed_parts_vs_oracle(parts, W):
    """Prefill with a ring (start > 0), decode steps and prefills straddling the ring, against the oracle."""
    dev = _dev()
    from heimdall_b200 import BifrostLayer
    H, G, D, d, S = 24, 4, 256, 128, 4
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=7)
    T = sum(parts)
    x, q, k, v, qr, kr = _layer_inputs(H, G, D, d, T, seed=11)
    f = lambda z: z.float()
    L = BifrostLayer.from_params(p, dev)
    cache_r, cache, s = {}, {}, 0
    for n in parts:
        sl = slice(s, s + n)
        o_ref = ob.student(p, f(x[:, sl]), f(q[:, sl]), f(k[:, sl]), f(v[:, sl]), f(qr[:, :, sl]), f(kr[:, :, sl]),
                           s, cache_r)
        o = L.student(x[:, sl].to(dev), q[:, sl].to(dev), k[:, sl].to(dev), v[:, sl].to(dev), qr[:, :, sl].to(dev),
                      kr[:, :, sl].to(dev), s, cache)
        torch.cuda.synchronize()
        assert ob.rel_l2(o.cpu(), o_ref) < O_TOL, (s, n)
        s += n
    assert ob.rel_l2(cache["S"].cpu(), cache_r["S"]) < S_TOL
    assert torch.equal(cache["ring_pos"].cpu(), cache_r["ring_pos"])


@pytest.mark.parametrize("scale", [64.0, 512.0])
def test_layer_large_values_vs_oracle(scale):
    """Values as a real v_proj gives them (not normalised): v scaled up to 512 passes through the fp16 value
    operands of the window (P V) and the delta rule (u, v', state copies) within tolerance; prefill with a ring,
    then decode steps."""
    dev = _dev()
    from heimdall_b200 import BifrostLayer
    H, G, D, d, S, W = 24, 4, 256, 128, 4, 128
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=21)
    parts = (300, 1, 200, 1)
    x, q, k, v, qr, kr = _layer_inputs(H, G, D, d, sum(parts), seed=23)
    v = (v.float() * scale).to(torch.bfloat16)
    f = lambda z: z.float()
    L = BifrostLayer.from_params(p, dev)
    cache_r, cache, s = {}, {}, 0
    for n in parts:
        sl = slice(s, s + n)
        o_ref = ob.student(p, f(x[:, sl]), f(q[:, sl]), f(k[:, sl]), f(v[:, sl]), f(qr[:, :, sl]), f(kr[:, :, sl]),
                           s, cache_r, dtype=torch.float64)
        o = L.student(x[:, sl].to(dev), q[:, sl].to(dev), k[:, sl].to(dev), v[:, sl].to(dev), qr[:, :, sl].to(dev),
                      kr[:, :, sl].to(dev), s, cache)
        torch.cuda.synchronize()
        assert torch.isfinite(o).all()
        assert ob.rel_l2(o.cpu(), o_ref) < O_TOL, (s, n)
        s += n
    assert ob.rel_l2(cache["S"].cpu(), cache_r["S"]) < S_TOL


def test_batch_equals_single():
    """B=2 equals two B=1 runs (the reference's native multi-sequence check, done on the layer core)."""
    dev = _dev()
    from heimdall_b200 import BifrostLayer
    H, G, D, d, W, S, T = 24, 4, 256, 128, 128, 4, 400
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=9)
    x, q, k, v, qr, kr = (z.to(dev) for z in _layer_inputs(H, G, D, d, T, seed=5, B=2))
    L = BifrostLayer.from_params(p, dev)
    o2 = L.student(x, q, k, v, qr, kr, 0, None)
    for b in range(2):
        o1 = L.student(x[b:b + 1], q[b:b + 1], k[b:b + 1], v[b:b + 1], qr[b:b + 1], kr[b:b + 1], 0, None)
        assert ob.rel_l2(o1.cpu(), o2[b:b + 1].cpu()) < 1e-6


@pytest.mark.parametrize("B,T,chunk", [(1, 1500, 512), (2, 700, 256), (1, 2600, 512)])
def test_student_host_matches_oracle(B, T, chunk):
    """The host-buffer prefill (chunks over a carried cache, copies overlapped on three streams) gives the
    one-pass result: against the oracle, and the carried cache equals the one-pass cache."""
    dev = _dev()
    from heimdall_b200 import BifrostLayer
    H, G, D, d, W, S = 24, 4, 256, 128, 256, 4
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=13)
    x, q, k, v, qr, kr = _layer_inputs(H, G, D, d, T, seed=17, B=B)
    f = lambda z: z.float()
    L = BifrostLayer.from_params(p, dev)
    pinned = [z.contiguous().pin_memory() for z in (x, q, k, v, qr, kr)]
    cache_h = {}
    o = L.student_host(*pinned, 0, cache_h, chunk=chunk)
    assert not o.is_cuda and o.shape == (B, T, H, D)
    for b in range(B):
        cache_r = {}
        o_ref = ob.student(p, f(x[b:b + 1]), f(q[b:b + 1]), f(k[b:b + 1]), f(v[b:b + 1]), f(qr[b:b + 1]),
                           f(kr[b:b + 1]), 0, cache_r)
        assert ob.rel_l2(o[b:b + 1], o_ref) < O_TOL, b
        assert ob.rel_l2(cache_h["S"][b:b + 1].cpu(), cache_r["S"]) < S_TOL, b
    cache_d = {}
    L.student(*(z.to(dev) for z in (x, q, k, v, qr, kr)), 0, cache_d)
    torch.cuda.synchronize()
    for key in ("ring_k", "ring_v", "ring_pos", "sink_k", "sink_v"):
        assert torch.equal(cache_h[key].cpu(), cache_d[key].cpu()), key


def _varlen_inputs(lens, G, R, D, seed):
    gen = torch.Generator().manual_seed(seed)
    T = sum(lens)
    q = F.normalize(torch.randn(1, T, G, R, D, generator=gen), dim=-1) * D ** -0.5
    k = F.normalize(torch.randn(1, T, G, D, generator=gen), dim=-1)
    v = torch.randn(1, T, G, D, generator=gen)
    g = -torch.rand(1, T, G, generator=gen) * 0.05
    beta = torch.rand(1, T, G, generator=gen)
    s0 = torch.randn(len(lens), G, D, D, generator=gen) * 0.05
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    return q, k, v, g, beta, s0, cu


def test_varlen_matches_per_sequence_oracle():
    """Packed sequences (cu_seqlens): each sequence runs its own recurrence from its own state, including
    empty, one-token and chunk-boundary lengths."""
    dev = _dev()
    from heimdall_b200.functional import delta_rule_gqa
    lens = [1, 127, 0, 128, 129, 300, 5, 700]
    G, R, D = 4, 2, 256
    q, k, v, g, beta, s0, cu = _varlen_inputs(lens, G, R, D, seed=31)
    o, s = delta_rule_gqa(*(z.to(dev) for z in (q, k, v, g, beta)), 64, s0.to(dev), cu_seqlens=cu.to(dev))
    torch.cuda.synchronize()
    for i, n in enumerate(lens):
        a, b = int(cu[i]), int(cu[i + 1])
        if n == 0:
            assert ob.rel_l2(s[i].cpu(), s0[i]) < 1e-6
            continue
        o_ref, s_ref = ob.gdn_gqa(q[:, a:b], k[:, a:b], v[:, a:b], g[:, a:b], beta[:, a:b], 64, s0[i:i + 1],
                                  dtype=torch.float64)
        assert ob.rel_l2(o[:, a:b].cpu(), o_ref) < O_TOL, i
        assert ob.rel_l2(s[i:i + 1].cpu(), s_ref) < S_TOL, i


def test_varlen_config4_matches_separate_calls():
    """BASELINE config 4 shapes: 8 sequences, lengths round(exp U[ln 2048, ln 65536]) (seed 0), packed;
    the packed call equals one call per sequence (same chunking per sequence, so up to rounding)."""
    dev = _dev()
    from heimdall_b200.functional import delta_rule_gqa
    gen = torch.Generator().manual_seed(0)
    lens = torch.exp(torch.empty(8).uniform_(math.log(2048), math.log(65536), generator=gen)).round().long().tolist()
    G, R, D = 4, 2, 256
    q, k, v, g, beta, s0, cu = _varlen_inputs(lens, G, R, D, seed=0)
    to = lambda z: z.to(dev)
    o, s = delta_rule_gqa(to(q), to(k), to(v.to(torch.bfloat16)), to(g), to(beta), 64, to(s0), cu_seqlens=to(cu))
    for i in range(8):
        a, b = int(cu[i]), int(cu[i + 1])
        o1, s1 = delta_rule_gqa(to(q[:, a:b]), to(k[:, a:b]), to(v[:, a:b].to(torch.bfloat16)), to(g[:, a:b]),
                                to(beta[:, a:b]), 64, to(s0[i:i + 1]))
        assert ob.rel_l2(o[:, a:b].cpu(), o1.cpu()) < 1e-5, i
        assert ob.rel_l2(s[i:i + 1].cpu(), s1.cpu()) < 1e-5, i

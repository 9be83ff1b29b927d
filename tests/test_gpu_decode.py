"""GPU parity: decode state update, memory-input projections (tcgen05), fused layer decode step.

Each CUDA result is compared with the CPU oracle (``oracle/bifrost_oracle.py``) on the same seeded,
bf16-valued inputs.  Tolerances (north star): outputs rel-L2 <= 2e-3, states rel-L2 <= 1e-3.
"""
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


@pytest.mark.parametrize("B,H,D", [(3, 4, 256), (2, 2, 64), (5, 3, 32)])
def test_delta_rule_step_matches_oracle(B, H, D):
    dev = _dev()
    import heimdall_b200 as hb
    g_ = torch.Generator().manual_seed(B * 100 + D)
    q = F.normalize(torch.randn(B, H, D, generator=g_), dim=-1) * D ** -0.5
    k = F.normalize(torch.randn(B, H, D, generator=g_), dim=-1)
    v = torch.randn(B, H, D, generator=g_)
    g = -torch.rand(B, H, generator=g_)
    beta = torch.rand(B, H, generator=g_)
    s0 = torch.randn(B, H, D, D, generator=g_) * 0.1
    o_ref, s_ref = ob.gdn_step(q, k, v, g, beta, s0, dtype=torch.float64)
    o, s = hb.delta_rule_step(*(z.to(dev) for z in (q, k, v, g, beta, s0)))
    torch.cuda.synchronize()
    assert ob.rel_l2(o.cpu(), o_ref) < 1e-5 and ob.rel_l2(s.cpu(), s_ref) < 1e-5


def test_delta_rule_step_golden(golden_gdn):
    """The reference's own delta_rule_step outputs (D=16 padded into a D=32 state with zeros)."""
    dev = _dev()
    import heimdall_b200 as hb
    c = golden_gdn["gdn_step"]
    pad = lambda z, n: F.pad(z, (0, n))
    q, k, v = pad(c["q"], 16), pad(c["k"], 16), pad(c["v"], 16)
    s0 = F.pad(c["s0"], (0, 16, 0, 16))
    o, s = hb.delta_rule_step(*(z.to(dev) for z in (q, k, v, c["g"], c["beta"], s0)))
    assert (o.cpu()[..., :16] - c["o"]).abs().max() < 1e-5
    assert (s.cpu()[..., :16, :16] - c["S"]).abs().max() < 1e-5


def test_gqa_step_in_place_bf16_values():
    dev = _dev()
    import heimdall_b200 as hb
    B, G, R, D = 4, 4, 6, 256
    g_ = torch.Generator().manual_seed(7)
    q = F.normalize(torch.randn(B, G, R, D, generator=g_), dim=-1) * D ** -0.5
    k = F.normalize(torch.randn(B, G, D, generator=g_), dim=-1)
    v = torch.randn(B, G, D, generator=g_).to(torch.bfloat16)
    g, beta = -torch.rand(B, G, generator=g_), torch.rand(B, G, generator=g_)
    s0 = torch.randn(B, G, D, D, generator=g_) * 0.1
    rep = lambda z: z.repeat_interleave(R, 1)
    o_ref, s_ref = ob.gdn_step(q.reshape(B, G * R, D), rep(k), rep(v.float()), rep(g), rep(beta),
                               s0.repeat_interleave(R, 1), dtype=torch.float64)
    S = s0.to(dev)
    o, s = hb.delta_rule_step_gqa(q.to(dev), k.to(dev), v.to(dev), g.to(dev), beta.to(dev), S, out_state=S)
    assert s.data_ptr() == S.data_ptr()
    assert ob.rel_l2(o.cpu().reshape(B, G * R, D), o_ref) < 1e-5
    assert ob.rel_l2(S.cpu(), s_ref[:, ::R]) < 1e-5


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


@pytest.mark.parametrize("T,d,B", [(200, 128, 2), (64, 5120, 1), (1, 256, 5)])
def test_mem_inputs_matches_oracle(T, d, B):
    """Projections on tcgen05: qm/km within fp16-weight rounding, g/beta/mix(x) near fp32."""
    dev = _dev()
    from heimdall_b200 import BifrostLayer
    H, G, D = 24, 4, 256
    p = layer_params(H, G, D, d, window=16, sinks=4, archival=1, seed=3)
    x, q, k, *_ = _layer_inputs(H, G, D, d, T, seed=11, B=B)
    start = 2
    pos = torch.arange(start, start + T)
    qm_r, km_r, g_r, b_r = ob.mem_inputs(p, x.float(), q.float(), k.float(), pos, dtype=torch.float64)
    mix_r = x.double() @ p.mix_w.double().t() + p.mix_b.double()
    L = BifrostLayer.from_params(p, dev)
    qm, km, g, beta, mixx = L.mem_inputs(x.to(dev), q.to(dev), k.to(dev), pos0=start)
    torch.cuda.synchronize()
    assert ob.rel_l2(qm.cpu(), qm_r) < 1e-3
    assert ob.rel_l2(km.cpu(), km_r) < 1e-3
    assert ob.rel_l2(g.cpu(), g_r) < 1e-4
    assert ob.rel_l2(beta.cpu(), b_r) < 1e-4
    assert ob.rel_l2(mixx.cpu(), mix_r) < 1e-4


def _cache_to(cache, dev):
    out = {}
    for k_, v_ in cache.items():
        if k_ in ("ring_k", "ring_v", "sink_k", "sink_v"):
            out[k_] = v_.to(device=dev, dtype=torch.bfloat16)
        else:
            out[k_] = v_.to(dev)
    return out


@pytest.mark.parametrize("memory", [True, False])
def test_layer_decode_matches_oracle(memory):
    """Prefill 40 tokens with the oracle (CPU), then decode 12 tokens on the GPU one by one."""
    dev = _dev()
    from heimdall_b200 import BifrostLayer
    H, G, D, d, W, S = 24, 4, 256, 128, 16, 4
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=5)
    T0, n = 40, 12
    x, q, k, v, qr, kr = _layer_inputs(H, G, D, d, T0 + n, seed=13, B=2)
    f = lambda z: z.float()
    cache = {}
    ob.student(p, f(x[:, :T0]), f(q[:, :T0]), f(k[:, :T0]), f(v[:, :T0]), f(qr[:, :, :T0]), f(kr[:, :, :T0]), 0,
               cache, memory=memory)
    gcache = _cache_to(cache, dev)
    L = BifrostLayer.from_params(p, dev)
    for i in range(T0, T0 + n):
        sl = slice(i, i + 1)
        o_ref = ob.student(p, f(x[:, sl]), f(q[:, sl]), f(k[:, sl]), f(v[:, sl]), f(qr[:, :, sl]), f(kr[:, :, sl]), i,
                           cache, memory=memory)
        o = L.student(x[:, sl].to(dev), q[:, sl].to(dev), k[:, sl].to(dev), v[:, sl].to(dev), qr[:, :, sl].to(dev),
                      kr[:, :, sl].to(dev), i, gcache, memory=memory)
        torch.cuda.synchronize()
        assert ob.rel_l2(o.cpu(), o_ref) < O_TOL, i
    if memory:
        assert ob.rel_l2(gcache["S"].cpu(), cache["S"]) < S_TOL
    assert torch.equal(gcache["ring_pos"].cpu(), cache["ring_pos"])
    assert torch.equal(gcache["ring_k"].cpu().float(), cache["ring_k"].float())
    assert ob.rel_l2(gcache["ring_km"].cpu(), cache["ring_km"]) < 1e-3
    assert ob.rel_l2(gcache["ring_g"].cpu(), cache["ring_g"]) < 1e-4


def test_layer_decode_early_positions_sinks():
    """Decode from position 0 (sinks fill up, memory inactive until W) against the oracle."""
    dev = _dev()
    from heimdall_b200 import BifrostLayer
    H, G, D, d, W, S = 24, 4, 256, 64, 8, 4
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=6)
    n = 20
    x, q, k, v, qr, kr = _layer_inputs(H, G, D, d, n, seed=17, B=1)
    f = lambda z: z.float()
    cache = {}
    # the first token goes through the oracle to create the ring (the GPU prefill path covers t > 1)
    ob.student(p, f(x[:, :1]), f(q[:, :1]), f(k[:, :1]), f(v[:, :1]), f(qr[:, :, :1]), f(kr[:, :, :1]), 0, cache)
    gcache = _cache_to(cache, dev)
    L = BifrostLayer.from_params(p, dev)
    for i in range(1, n):
        sl = slice(i, i + 1)
        o_ref = ob.student(p, f(x[:, sl]), f(q[:, sl]), f(k[:, sl]), f(v[:, sl]), f(qr[:, :, sl]), f(kr[:, :, sl]), i,
                           cache)
        o = L.student(x[:, sl].to(dev), q[:, sl].to(dev), k[:, sl].to(dev), v[:, sl].to(dev), qr[:, :, sl].to(dev),
                      kr[:, :, sl].to(dev), i, gcache)
        assert ob.rel_l2(o.cpu(), o_ref) < O_TOL, i
    assert gcache["sink_k"].shape == cache["sink_k"].shape
    assert ob.rel_l2(gcache["S"].cpu(), cache["S"]) < S_TOL


def test_layer_decode_graph_replay_matches_eager():
    """The fused decode step captured in a CUDA graph (its gate projections run on a forked stream inside the
    capture) leaves the same outputs and cache as the same step run eagerly."""
    dev = _dev()
    from heimdall_b200 import BifrostLayer, _lib
    from heimdall_b200.functional import ptr
    from heimdall_b200.layer import ctypes_ref
    from heimdall_b200.structs import BfRingCache
    H, G, D, d, W, S = 24, 4, 256, 128, 16, 4
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=5)
    T0, B = 40, 2
    x, q, k, v, qr, kr = _layer_inputs(H, G, D, d, T0 + 1, seed=13, B=B)
    f = lambda z: z.float()
    cache = {}
    ob.student(p, f(x[:, :T0]), f(q[:, :T0]), f(k[:, :T0]), f(v[:, :T0]), f(qr[:, :, :T0]), f(kr[:, :, :T0]), 0,
               cache)
    L = BifrostLayer.from_params(p, dev)
    step = [z.to(dev).contiguous() for z in (x[:, T0], q[:, T0], k[:, T0], v[:, T0], qr[:, :, T0], kr[:, :, T0])]
    pos = torch.full((B,), T0, dtype=torch.int64, device=dev)
    nws = _lib.size("bf_layer_decode_workspace", B, H, G, D, W)

    def make():
        c = _cache_to(cache, dev)
        st = BfRingCache(ptr(c["ring_k"]), ptr(c["ring_v"]), ptr(c["ring_km"]), ptr(c["ring_g"]), ptr(c["ring_beta"]),
                         ptr(c["ring_pos"]), 0, ptr(c["sink_k"]), ptr(c["sink_v"]), S, ptr(c["S"]))
        return c, st, torch.empty(B, H, D, device=dev), torch.empty(nws, dtype=torch.uint8, device=dev)

    def call(st, o, ws, stream):
        _lib.call("bf_bifrost_layer_decode", ctypes_ref(L.struct), *(ptr(z) for z in step), ptr(pos), B,
                  ctypes_ref(st), 1, ptr(o), 0, ptr(ws), ws.numel(), stream)

    ca, sta, oa, wsa = make()
    call(sta, oa, wsa, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    cb, stb, ob_, wsb = make()
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        call(stb, ob_, wsb, s.cuda_stream)
    graph.replay()
    torch.cuda.synchronize()
    assert ob.rel_l2(ob_.cpu(), oa.cpu()) < 1e-6
    for key in ("S", "ring_km", "ring_g", "ring_beta"):
        assert ob.rel_l2(cb[key].cpu(), ca[key].cpu()) < 1e-6, key
    assert torch.equal(cb["ring_k"].cpu(), ca["ring_k"].cpu()) and torch.equal(cb["ring_pos"].cpu(), ca["ring_pos"].cpu())
    del graph


def test_two_devices_in_one_process():
    """The kernels' shared-memory opt-ins and per-device state are per device: a decode state step and a
    layer prefill on device 0, then the same on device 1 of the same process, both match the oracle."""
    _dev()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import heimdall_b200 as hb
    from heimdall_b200 import BifrostLayer
    H, G, D, d, W, S, T = 24, 4, 256, 128, 64, 4, 300
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=23)
    x, q, k, v, qr, kr = _layer_inputs(H, G, D, d, T, seed=29)
    f = lambda z: z.float()
    o_ref = ob.student(p, f(x), f(q), f(k), f(v), f(qr), f(kr), 0, None)
    g_ = torch.Generator().manual_seed(5)
    qs = F.normalize(torch.randn(2, G, D, generator=g_), dim=-1) * D ** -0.5
    ks = F.normalize(torch.randn(2, G, D, generator=g_), dim=-1)
    vs, gs, bs = torch.randn(2, G, D, generator=g_), -torch.rand(2, G, generator=g_), torch.rand(2, G, generator=g_)
    s0 = torch.randn(2, G, D, D, generator=g_) * 0.1
    os_ref, ss_ref = ob.gdn_step(qs, ks, vs, gs, bs, s0, dtype=torch.float64)
    for i in (0, 1):
        dev = torch.device("cuda", i)
        with torch.cuda.device(dev):
            o_s, s_s = hb.delta_rule_step(*(z.to(dev) for z in (qs, ks, vs, gs, bs, s0)))
            L = BifrostLayer.from_params(p, dev)
            o = L.student(*(z.to(dev) for z in (x, q, k, v, qr, kr)), 0, None)
            torch.cuda.synchronize(dev)
        assert ob.rel_l2(o_s.cpu(), os_ref) < 1e-5 and ob.rel_l2(s_s.cpu(), ss_ref) < 1e-5, i
        assert ob.rel_l2(o.cpu(), o_ref) < O_TOL, i

"""GPU parity at the production geometry of the Bifrost layer: window W = 2048 with
4 sinks, hidden size d = 5120, decode batches with per-sequence positions spread over 4K-128K, and the
delta-rule state over 131072 tokens with an archival (never-forgetting) head.

These are the sizes the bench runs.  Every comparison is against the CPU oracle (``oracle/bifrost_oracle.py``,
a restatement of the reference's PyTorch path pinned to the reference's own outputs) on the same seeded,
bf16-valued inputs.  Tolerances (north star): outputs rel-L2 <= 2e-3, states rel-L2 <= 1e-3, max abs lse
error <= 1e-3; ring entries bit-exact where they are copies (keys, values, positions).

At W = 2048 the window kernels run their production paths: 16-17 key tiles per query tile with the band edge
inside a tile (prefill), and four 512-slot splits per (sequence, KV head) merged with the sinks and the new
token by the combine kernel (decode).
"""
import math

import pytest
import torch
import torch.nn.functional as F

from oracle import bifrost_oracle as ob
from params import layer_params

pytestmark = pytest.mark.gpu

O_TOL, S_TOL, LSE_TOL = 2e-3, 1e-3, 1e-3
H, G, D, W, S = 24, 4, 256, 2048, 4
R = H // G


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


def _rms(z):
    return z * torch.rsqrt(z.square().mean(-1, keepdim=True) + 1e-6)


def _bf(z):
    return z.to(torch.bfloat16)


def _threads():
    torch.set_num_threads(max(1, torch.get_num_threads()))


# ------------------------------------------------------------------------------------------------ window prefill
@pytest.mark.parametrize("T,start", [(4999, 0), (3001, 10000)])
def test_window_prefill_w2048(T, start):
    """Window + sinks attention at W = 2048: from an empty cache (start 0, the sinks are the first tokens) and
    with a full ring (start > W: the W ring rows in time order ahead of the new tokens)."""
    dev = _dev()
    _threads()
    import heimdall_b200 as hb
    B = 1
    gen = torch.Generator().manual_seed(T + start)
    nring = W if start > 0 else 0
    Tk = nring + T
    qr = _bf(_rms(torch.randn(B, H, T, D, generator=gen)))
    ek = _bf(_rms(torch.randn(B, G, Tk, D, generator=gen)))
    ev = _bf(_rms(torch.randn(B, G, Tk, D, generator=gen)))
    if start == 0:
        sk, sv = ek[:, :, :S].contiguous(), ev[:, :, :S].contiguous()
    else:
        sk, sv = _bf(_rms(torch.randn(B, G, S, D, generator=gen))), _bf(_rms(torch.randn(B, G, S, D, generator=gen)))
    pos = torch.arange(start, start + T)
    kpos0 = start - nring
    ext_pos = torch.arange(kpos0, kpos0 + Tk)
    ok_, ov_, op_ = ek.float(), ev.float(), ext_pos
    if nring == 0:   # the reference's ext layout always has W ring rows ahead; empty ones have position -1
        ok_ = torch.cat((ok_.new_zeros(B, G, W, D), ok_), 2)
        ov_ = torch.cat((ov_.new_zeros(B, G, W, D), ov_), 2)
        op_ = torch.cat((torch.full((W,), -1, dtype=torch.long), op_))
    o_ref, lse_ref = ob.window_attention(qr.float(), ok_, ov_, op_, sk.float(), sv.float(), pos, W, S, block=256)
    o, lse = hb.window_attention(qr.to(dev), ek.to(dev), ev.to(dev), start, kpos0, S, W, sk.to(dev), sv.to(dev))
    torch.cuda.synchronize()
    assert ob.rel_l2(o.cpu(), o_ref) < O_TOL
    assert float((lse.cpu().double() - lse_ref.double()).abs().max()) < LSE_TOL


# ------------------------------------------------------------------------------------------------ layer prefill
def _layer_inputs(d, T, seed, B=1):
    gen = torch.Generator().manual_seed(seed)
    x = _bf(torch.randn(B, T, d, generator=gen))
    q = _bf(_rms(torch.randn(B, T, H, D, generator=gen)))
    k = _bf(_rms(torch.randn(B, T, G, D, generator=gen)))
    v = _bf(_rms(torch.randn(B, T, G, D, generator=gen)))
    qr = _bf(_rms(torch.randn(B, H, T, D, generator=gen)))
    kr = _bf(_rms(torch.randn(B, G, T, D, generator=gen)))
    return x, q, k, v, qr, kr


def test_layer_prefill_d5120_w2048_parts():
    """The fused layer at d = 5120, W = 2048: a 6000-token prefill from an empty cache, then a 2500-token
    prefill from the ring it left, then two decode tokens; outputs, state and ring against the oracle."""
    dev = _dev()
    _threads()
    from heimdall_b200 import BifrostLayer
    d = 5120
    parts = (6000, 2500, 1, 1)
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=31)
    x, q, k, v, qr, kr = _layer_inputs(d, sum(parts), seed=32)
    f = lambda z: z.float()
    L = BifrostLayer.from_params(p, dev)
    cache_r, cache, s = {}, {}, 0
    for n in parts:
        sl = slice(s, s + n)
        with torch.no_grad():
            o_ref = ob.student(p, f(x[:, sl]), f(q[:, sl]), f(k[:, sl]), f(v[:, sl]), f(qr[:, :, sl]),
                               f(kr[:, :, sl]), s, cache_r)
        o = L.student(x[:, sl].to(dev), q[:, sl].to(dev), k[:, sl].to(dev), v[:, sl].to(dev),
                      qr[:, :, sl].contiguous().to(dev), kr[:, :, sl].contiguous().to(dev), s, cache)
        torch.cuda.synchronize()
        assert ob.rel_l2(o.cpu(), o_ref) < O_TOL, (s, n)
        s += n
    assert ob.rel_l2(cache["S"].cpu(), cache_r["S"]) < S_TOL
    assert torch.equal(cache["ring_pos"].cpu(), cache_r["ring_pos"])
    assert torch.equal(cache["ring_k"].cpu().float(), cache_r["ring_k"].float())
    assert torch.equal(cache["ring_v"].cpu().float(), cache_r["ring_v"].float())
    assert ob.rel_l2(cache["ring_km"].cpu(), cache_r["ring_km"]) < 1e-3
    assert ob.rel_l2(cache["ring_g"].cpu(), cache_r["ring_g"]) < 1e-4
    assert ob.rel_l2(cache["ring_beta"].cpu(), cache_r["ring_beta"]) < 1e-4


# ------------------------------------------------------------------------------------------------ decode
def _decode_cache(B, pos, gen):
    """A filled decode cache per sequence: the W ring entries before each position (slot = position mod W),
    4 sinks, a state; values generated as in BASELINE config 2."""
    ring_abs = pos[:, None] - W + torch.arange(W)[None]                         # [B, W] positions p-W .. p-1
    ring_pos = torch.empty(B, W, dtype=torch.long).scatter_(1, ring_abs % W, ring_abs)
    return dict(ring_k=_bf(_rms(torch.randn(B, G, W, D, generator=gen))),
                ring_v=_bf(_rms(torch.randn(B, G, W, D, generator=gen))),
                ring_km=F.normalize(torch.randn(B, W, G, D, generator=gen), dim=-1),
                ring_g=-torch.rand(B, W, G, generator=gen) * 0.01,
                ring_beta=torch.rand(B, W, G, generator=gen), ring_pos=ring_pos,
                sink_k=_bf(_rms(torch.randn(B, G, S, D, generator=gen))),
                sink_v=_bf(_rms(torch.randn(B, G, S, D, generator=gen))),
                S=torch.randn(B, G, D, D, generator=gen) * 0.02)


def _oracle_cache(c, b):
    """Sequence b of a batched cache as the reference's per-sequence dict (B = 1, ring_pos [W], fp32 values)."""
    out = {}
    for key, t in c.items():
        t = t[b:b + 1].clone()
        out[key] = t[0] if key == "ring_pos" else (t.float() if t.is_floating_point() else t)
    return out


@pytest.mark.parametrize("memory", [True, False])
def test_layer_decode_w2048_per_sequence_positions(memory):
    """Decode at W = 2048 (four 512-slot splits and the combine), d = 5120, B = 8 sequences at their own
    positions in [4096, 131072) with a per-sequence [B, W] ring_pos, three steps.  Two sequences sit on ring
    boundaries: one evicts slot 0 at the first step (p mod W == 0), one writes the last slot (p mod W == W-1)
    and then wraps to slot 0.  Each sequence is checked against the oracle run on it alone."""
    dev = _dev()
    _threads()
    from heimdall_b200 import BifrostLayer
    d, B, steps = 5120, 8, 3
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=41)
    gen = torch.Generator().manual_seed(42)
    pos = torch.randint(4096, 131072, (B,), generator=gen)
    pos[0] = 40 * W                 # evicts slot 0 first
    pos[1] = 20 * W + W - 1         # writes slot W-1, then slot 0
    pos[2] = 4096
    c = _decode_cache(B, pos, gen)
    ref = [_oracle_cache(c, b) for b in range(B)]
    gc = {key: t.to(dev) for key, t in c.items()}
    L = BifrostLayer.from_params(p, dev)
    lse = torch.empty(B, H, device=dev)
    for step in range(steps):
        x = _bf(torch.randn(B, d, generator=gen))
        q = _bf(_rms(torch.randn(B, H, D, generator=gen)))
        k = _bf(_rms(torch.randn(B, G, D, generator=gen)))
        v = _bf(_rms(torch.randn(B, G, D, generator=gen)))
        qr = _bf(_rms(torch.randn(B, H, D, generator=gen)))
        kr = _bf(_rms(torch.randn(B, G, D, generator=gen)))
        o = L.decode_step(x.to(dev), q.to(dev), k.to(dev), v.to(dev), qr.to(dev), kr.to(dev), pos.to(dev), gc,
                          memory=memory, lse=lse)
        torch.cuda.synchronize()
        for b in range(B):
            pb = int(pos[b])
            f = lambda z: z[b:b + 1].float()
            o_ref = ob.student(p, f(x)[:, None], f(q)[:, None], f(k)[:, None], f(v)[:, None], f(qr)[:, :, None],
                               f(kr)[:, :, None], pb, ref[b], memory=memory)
            assert ob.rel_l2(o[b].cpu(), o_ref[0, 0]) < O_TOL, (step, b, pb)
        pos += 1
    for b in range(B):
        assert torch.equal(gc["ring_pos"][b].cpu(), ref[b]["ring_pos"]), b
        assert torch.equal(gc["ring_k"][b].cpu().float(), ref[b]["ring_k"][0]), b
        assert torch.equal(gc["ring_v"][b].cpu().float(), ref[b]["ring_v"][0]), b
        assert ob.rel_l2(gc["ring_km"][b].cpu(), ref[b]["ring_km"][0]) < 1e-3, b
        assert ob.rel_l2(gc["ring_g"][b].cpu(), ref[b]["ring_g"][0]) < 1e-4, b
        if memory:
            assert ob.rel_l2(gc["S"][b].cpu(), ref[b]["S"][0]) < S_TOL, b


def test_decode_bench_batch_64_sequences():
    """The bench's decode batch (64 sequences, W = 2048, d = 5120) for one step, checked
    on a sample of sequences against the oracle, with the window log-sum-exp."""
    dev = _dev()
    _threads()
    from heimdall_b200 import BifrostLayer
    d, B = 5120, 64
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=43)
    gen = torch.Generator().manual_seed(44)
    pos = torch.randint(4096, 131072, (B,), generator=gen)
    c = _decode_cache(B, pos, gen)
    gc = {key: t.to(dev) for key, t in c.items()}
    L = BifrostLayer.from_params(p, dev)
    x = _bf(torch.randn(B, d, generator=gen))
    q, qr = _bf(_rms(torch.randn(B, H, D, generator=gen))), _bf(_rms(torch.randn(B, H, D, generator=gen)))
    k, kr = _bf(_rms(torch.randn(B, G, D, generator=gen))), _bf(_rms(torch.randn(B, G, D, generator=gen)))
    v = _bf(_rms(torch.randn(B, G, D, generator=gen)))
    lse = torch.empty(B, H, device=dev)
    o = L.decode_step(*(z.to(dev) for z in (x, q, k, v, qr, kr)), pos.to(dev), gc, lse=lse)
    torch.cuda.synchronize()
    for b in (0, 17, 33, 63):
        rb = _oracle_cache(c, b)
        f = lambda z: z[b:b + 1].float()
        pb = int(pos[b])
        o_ref = ob.student(p, f(x)[:, None], f(q)[:, None], f(k)[:, None], f(v)[:, None], f(qr)[:, :, None],
                           f(kr)[:, :, None], pb, rb)
        assert ob.rel_l2(o[b].cpu(), o_ref[0, 0]) < O_TOL, b
        assert ob.rel_l2(gc["S"][b].cpu(), rb["S"][0]) < S_TOL, b
        # the window lse of the new token, from the oracle's window over the same keys
        slots = torch.arange(pb - W, pb) % W
        ek = torch.cat((c["ring_k"][b:b + 1, :, slots].float(), kr[b:b + 1, :, None].float()), 2)
        ev = torch.cat((c["ring_v"][b:b + 1, :, slots].float(), v[b:b + 1, :, None].float()), 2)
        ep = torch.cat((c["ring_pos"][b, slots], torch.tensor([pb])))
        _, lse_ref = ob.window_attention(qr[b:b + 1, :, None].float(), ek, ev, ep, c["sink_k"][b:b + 1].float(),
                                         c["sink_v"][b:b + 1].float(), torch.tensor([pb]), W, S)
        assert float((lse[b].cpu() - lse_ref[0, :, 0]).abs().max()) < LSE_TOL, b


# ------------------------------------------------------------------------------------------------ long state
def test_delta_rule_long_state_archival():
    """The delta rule alone over T = 131072 tokens (BASELINE config 3 length) with fixed decays of half-lives
    2048 .. 1M tokens and the last head archival (alpha = 1, never forgets, as in config 4), against the
    chunked oracle in float64.  The GPU scan feeds fp16 copies of the state to the tensor core once per
    128-token chunk (1024 times here); the final state must stay within 1e-3 and the outputs within 2e-3."""
    dev = _dev()
    _threads()
    import heimdall_b200 as hb
    T, Gh = 131072, 4
    gen = torch.Generator().manual_seed(51)
    q = F.normalize(torch.randn(1, T, Gh, D, generator=gen), dim=-1) * D ** -0.5
    k = F.normalize(torch.randn(1, T, Gh, D, generator=gen), dim=-1)
    v = _bf(torch.randn(1, T, Gh, D, generator=gen)).float()
    beta = torch.sigmoid(torch.randn(1, T, Gh, generator=gen))
    life = torch.logspace(math.log10(2048), 6.0, Gh)
    g = (-(math.log(2.0) / life)).expand(1, T, Gh).contiguous()
    g[..., -1] = 0.0
    o, s = hb.delta_rule(q.to(dev), k.to(dev), v.to(dev), g.to(dev), beta.to(dev))
    torch.cuda.synchronize()
    o, s = o.cpu(), s.cpu()
    with torch.no_grad():
        o_ref, s_ref = ob.gdn_chunked(q, k, v, g, beta, 128, None, dtype=torch.float64)
    for h in range(Gh):
        es = ob.rel_l2(s[:, h], s_ref[:, h])
        assert es < S_TOL, (h, es)
    assert ob.rel_l2(o, o_ref) < O_TOL
    # the last 4096 tokens alone (where the accumulated state error would show most)
    assert ob.rel_l2(o[:, -4096:], o_ref[:, -4096:]) < O_TOL


def test_layer_prefill_split_window_pieces():
    """Prefills long enough for the window to run as several launches with the memory reads of each finished
    piece beside the next (4 pieces here: 9000 tokens from an empty cache, then 5000 more from the ring), against
    the oracle; outputs, state and ring."""
    dev = _dev()
    _threads()
    from heimdall_b200 import BifrostLayer
    d, Wl = 128, 512
    parts = (9000, 5000)
    p = layer_params(H, G, D, d, window=Wl, sinks=S, archival=1, seed=71)
    x, q, k, v, qr, kr = _layer_inputs(d, sum(parts), seed=72)
    f = lambda z: z.float()
    L = BifrostLayer.from_params(p, dev)
    cache_r, cache, s = {}, {}, 0
    for n in parts:
        sl = slice(s, s + n)
        with torch.no_grad():
            o_ref = ob.student(p, f(x[:, sl]), f(q[:, sl]), f(k[:, sl]), f(v[:, sl]), f(qr[:, :, sl]),
                               f(kr[:, :, sl]), s, cache_r)
        o = L.student(x[:, sl].to(dev), q[:, sl].to(dev), k[:, sl].to(dev), v[:, sl].to(dev),
                      qr[:, :, sl].contiguous().to(dev), kr[:, :, sl].contiguous().to(dev), s, cache)
        torch.cuda.synchronize()
        assert ob.rel_l2(o.cpu(), o_ref) < O_TOL, (s, n)
        s += n
    assert ob.rel_l2(cache["S"].cpu(), cache_r["S"]) < S_TOL
    assert torch.equal(cache["ring_pos"].cpu(), cache_r["ring_pos"])

"""GPU parity of the llama.cpp state-row interchange (``bf_llama_state_pack`` / ``bf_llama_state_unpack``).

Pack and unpack are layout copies, so they must equal the CPU oracle (``oracle/llama_state.py``) bit for bit:
on caches the GPU prefill built, on production-geometry decode caches (W = 2048, per-sequence positions, a
sequence still inside its sinks), and on arbitrary rows (unpack's bf16 rounding included).  The last test
continues a sequence across the boundary: the GPU decode of a cache, packed, must match the port's decode
graph (restated in the oracle) run on the row packed before the step.
"""
import pytest
import torch
import torch.nn.functional as F

from oracle import bifrost_oracle as ob
from oracle import llama_state as ls
from params import layer_params

pytestmark = pytest.mark.gpu

O_TOL = 2e-3
H, G, D, S = 24, 4, 256, 4
R = H // G


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


def _rms(z):
    return z * torch.rsqrt(z.square().mean(-1, keepdim=True) + 1e-6)


def _bf(z):
    return z.to(torch.bfloat16)


def _inputs(B, t, d, gen):
    n = lambda *s: torch.randn(*s, generator=gen)
    return (_bf(n(B, t, d)), _bf(_rms(n(B, t, H, D))), _bf(_rms(n(B, t, G, D))), _bf(_rms(n(B, t, G, D))),
            _bf(_rms(n(B, H, t, D))), _bf(_rms(n(B, G, t, D))))


def _cpu(cache):
    return {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in cache.items()}


@pytest.mark.parametrize("T0", [3, 40, 64, 100, 200])
def test_pack_after_gpu_prefill_matches_oracle(T0):
    dev = _dev()
    from heimdall_b200 import BifrostLayer
    from heimdall_b200.interchange import pack_llama_state, unpack_llama_state
    W, d, B = 64, 128, 2
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=60)
    L = BifrostLayer.from_params(p, dev)
    gen = torch.Generator().manual_seed(T0)
    x, q, k, v, qr, kr = (z.to(dev) for z in _inputs(B, T0, d, gen))
    cache = {}
    L.student(x, q, k, v, qr, kr, 0, cache)
    rows = pack_llama_state(L, cache, T0)
    torch.cuda.synchronize()
    ref = ls.pack(_cpu(cache), [T0] * B, G, D, W, S)
    assert torch.equal(rows.cpu(), ref)
    back = unpack_llama_state(L, rows, T0, per_seq_pos=False)
    torch.cuda.synchronize()
    for key in ("ring_k", "ring_v", "ring_km", "ring_g", "ring_beta", "ring_pos", "sink_k", "sink_v"):
        assert torch.equal(back[key].cpu(), cache[key].cpu()), key
    if "S" in cache:
        assert torch.equal(back["S"].cpu(), cache["S"].cpu())
    else:
        assert not back["S"].any()


def _decode_cache(B, pos, W, gen):
    ring_abs = pos[:, None] - W + torch.arange(W)[None]
    ring_pos = torch.empty(B, W, dtype=torch.long).scatter_(1, ring_abs % W, ring_abs)
    ring_pos = torch.where(ring_pos >= 0, ring_pos, torch.full_like(ring_pos, -1))
    return dict(ring_k=_bf(_rms(torch.randn(B, G, W, D, generator=gen))),
                ring_v=_bf(_rms(torch.randn(B, G, W, D, generator=gen))),
                ring_km=F.normalize(torch.randn(B, W, G, D, generator=gen), dim=-1),
                ring_g=-torch.rand(B, W, G, generator=gen) * 0.01,
                ring_beta=torch.rand(B, W, G, generator=gen), ring_pos=ring_pos,
                sink_k=_bf(_rms(torch.randn(B, G, S, D, generator=gen))),
                sink_v=_bf(_rms(torch.randn(B, G, S, D, generator=gen))),
                S=torch.randn(B, G, D, D, generator=gen) * 0.02)


def test_pack_unpack_w2048_per_sequence_positions():
    """W = 2048, four sequences at their own positions (one past its ring wrap, one on the wrap, one inside
    its first window, one still inside its sinks), per-sequence ring_pos."""
    dev = _dev()
    from heimdall_b200 import BifrostLayer
    from heimdall_b200.interchange import llama_state_floats, pack_llama_state, unpack_llama_state
    W, d = 2048, 64
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=61)
    L = BifrostLayer.from_params(p, dev)
    gen = torch.Generator().manual_seed(61)
    pos = torch.tensor([70001, 2 * W, 1000, 3])
    B = pos.numel()
    c = _decode_cache(B, pos, W, gen)
    gc = {k: t.to(dev) for k, t in c.items()}
    n = llama_state_floats(G, D, W, S)
    assert n == ls.state_floats(G, D, W, S)
    rows = torch.full((B, n + 12), float("nan"), device=dev)      # padded row stride: every float is written
    pack_llama_state(L, gc, pos.to(dev), rows=rows)
    torch.cuda.synchronize()
    ref = ls.pack(c, pos.tolist(), G, D, W, S)
    assert torch.equal(rows[:, :n].cpu(), ref)
    assert torch.isnan(rows[:, n:]).all()
    back = unpack_llama_state(L, rows, pos.to(dev))
    torch.cuda.synchronize()
    assert torch.equal(back["ring_pos"].cpu(), c["ring_pos"])
    valid = c["ring_pos"] >= 0
    for key in ("ring_k", "ring_v"):
        got, want = back[key].cpu(), c[key]
        for b in range(B):
            assert torch.equal(got[b][:, valid[b]], want[b][:, valid[b]]), (key, b)
            assert not got[b][:, ~valid[b]].any(), (key, b)
    for key in ("ring_km", "ring_g", "ring_beta"):
        got, want = back[key].cpu(), c[key]
        for b in range(B):
            assert torch.equal(got[b][valid[b]], want[b][valid[b]]), (key, b)
    assert back["sink_k"].shape[2] == 3                                  # min(sinks, smallest next position)
    assert torch.equal(back["sink_k"].cpu(), c["sink_k"][:, :, :3])
    assert torch.equal(back["sink_v"].cpu(), c["sink_v"][:, :, :3])
    assert torch.equal(back["S"].cpu(), c["S"])


def test_unpack_arbitrary_rows_matches_oracle():
    """Rows written by another program (arbitrary fp32 values): unpack rounds k_rope/v to bf16 like the
    oracle, bit for bit, at per-sequence positions."""
    dev = _dev()
    from heimdall_b200 import BifrostLayer
    from heimdall_b200.interchange import unpack_llama_state
    W, d = 64, 64
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=0, seed=62)
    L = BifrostLayer.from_params(p, dev)
    gen = torch.Generator().manual_seed(62)
    pos = [5, 64, 65, 1000]
    rows = torch.randn(len(pos), ls.state_floats(G, D, W, S), generator=gen) * 3
    back = unpack_llama_state(L, rows.to(dev), torch.tensor(pos).to(dev))
    torch.cuda.synchronize()
    ref = ls.unpack(rows, pos, G, D, W, S)
    for key, want in ref.items():
        assert torch.equal(back[key].cpu(), want), key


def test_gpu_decode_continues_like_port_on_packed_row():
    """prefill (GPU) -> pack -> the port's decode of one token on the row (oracle) versus the GPU decode of the
    same token on the cache, then pack: same output and the same row (copies exact, fp32 fields to the decode
    tolerance)."""
    dev = _dev()
    from heimdall_b200 import BifrostLayer
    from heimdall_b200.interchange import pack_llama_state
    W, d, B, T0 = 64, 128, 2, 150
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=63)
    L = BifrostLayer.from_params(p, dev)
    gen = torch.Generator().manual_seed(63)
    x, q, k, v, qr, kr = (z.to(dev) for z in _inputs(B, T0, d, gen))
    cache = {}
    L.student(x, q, k, v, qr, kr, 0, cache)
    rows0 = pack_llama_state(L, cache, T0).cpu()
    x1, q1, k1, v1, qr1, kr1 = _inputs(B, 1, d, gen)
    cache["ring_pos"] = cache["ring_pos"][None].expand(B, W).contiguous()
    pos = torch.full((B,), T0, dtype=torch.int64)
    o = L.decode_step(x1[:, 0].to(dev), q1[:, 0].to(dev), k1[:, 0].to(dev), v1[:, 0].to(dev), qr1[:, :, 0].to(dev),
                      kr1[:, :, 0].to(dev), pos.to(dev), cache)
    rows1 = pack_llama_state(L, cache, T0 + 1).cpu()
    torch.cuda.synchronize()
    qm, km, g, beta = ob.mem_inputs(p, x1.float(), q1.float(), k1.float(), torch.tensor([T0]), dtype=torch.float64)
    mixx = x1.double() @ p.mix_w.double().t() + p.mix_b.double()
    GD = G * D
    for b in range(B):
        row = rows0[b].clone()
        new = dict(k_rope=kr1[b, :, 0].float(), v=v1[b, 0].float(), km=km[b, 0], g=g[b, 0], beta=beta[b, 0])
        o_port = ls.llama_decode(row, T0, new, qr1[b, :, 0].float(), qm[b, 0], mixx[b, 0], p.mix_lse, p.mem_scale,
                                 G, D, W, S)
        assert ob.rel_l2(o[b].cpu(), o_port) < O_TOL, b
        reg_g, kp_g, vp_g, dl_g = ls._views(rows1[b], G, D, W, S)
        reg_p, kp_p, vp_p, dl_p = ls._views(row, G, D, W, S)
        live = [l for l in range(S + W + 1) if l != ls.llama_slot(T0 + 1 - W - 1, W, S)]
        assert torch.equal(reg_g[live, :2 * GD], reg_p[live, :2 * GD]), b        # k_rope and v: copies
        assert torch.equal(kp_g[:, live], kp_p[:, live]) and torch.equal(vp_g[:, :, live], vp_p[:, :, live])
        assert ob.rel_l2(reg_g[live, 2 * GD:], reg_p[live, 2 * GD:]) < 1e-4, b   # k_mem, g, beta
        assert ob.rel_l2(dl_g, dl_p) < 1e-3, b                                    # the state after the step

"""BASELINE config 4 as the full layer: packed variable-length sequences through window + memory + gate, each
sequence with its own positions, sinks, ring and a memory state reset to zero at its start.

The reference has no packed form (no cu_seqlens anywhere); its semantics for a batch of sequences of
different lengths is ``HybridAttention._student`` run once per sequence (heimdall/hibrit.py:363-424).  The
oracle does exactly that, and the packed GPU result must match it sequence by sequence: outputs rel-L2 <= 2e-3,
final states rel-L2 <= 1e-3, ring positions and keys exact.
"""
import math

import pytest
import torch

from oracle import bifrost_oracle as ob
from params import layer_params

pytestmark = pytest.mark.gpu
O_TOL, S_TOL = 2e-3, 1e-3


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


def _inputs(H, G, D, d, T, seed):
    gen = torch.Generator().manual_seed(seed)
    rms = lambda z: z * torch.rsqrt(z.square().mean(-1, keepdim=True) + 1e-6)
    bf = lambda z: z.to(torch.bfloat16)
    return (bf(torch.randn(1, T, d, generator=gen)), bf(rms(torch.randn(1, T, H, D, generator=gen))),
            bf(rms(torch.randn(1, T, G, D, generator=gen))), bf(rms(torch.randn(1, T, G, D, generator=gen))),
            bf(rms(torch.randn(1, H, T, D, generator=gen))), bf(rms(torch.randn(1, G, T, D, generator=gen))))


def _check(p, lens, d, seed, memory=True):
    dev = _dev()
    from heimdall_b200 import BifrostLayer
    H, G, D = p.fq.shape[0], p.fk.shape[0], p.fq.shape[-1]
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    T = cu[-1]
    x, q, k, v, qr, kr = _inputs(H, G, D, d, T, seed)
    L = BifrostLayer.from_params(p, dev)
    caches = [{} for _ in lens]
    o = L.student_varlen(*(z.to(dev) for z in (x, q, k, v, qr, kr)), cu, memory=memory, caches=caches)
    torch.cuda.synchronize()
    f = lambda z: z.float()
    for i, (a, b) in enumerate(zip(cu, cu[1:])):
        if a == b:
            assert caches[i] == {}
            continue
        cr = {}
        o_ref = ob.student(p, f(x[:, a:b]), f(q[:, a:b]), f(k[:, a:b]), f(v[:, a:b]), f(qr[:, :, a:b]),
                           f(kr[:, :, a:b]), 0, cr, memory=memory)
        assert ob.rel_l2(o[:, a:b].cpu(), o_ref) < O_TOL, (i, b - a)
        assert torch.equal(caches[i]["ring_pos"].cpu(), cr["ring_pos"]), i
        assert torch.equal(caches[i]["ring_k"].cpu().float(), cr["ring_k"].float()), i
        if memory and "S" in cr:
            assert ob.rel_l2(caches[i]["S"].cpu(), cr["S"]) < S_TOL, i


@pytest.mark.parametrize("memory", [True, False])
def test_varlen_layer_small_window(memory):
    """Ragged lengths around the window and the 128-token chunks, an empty and a one-token sequence."""
    H, G, D, d, W, S = 24, 4, 256, 128, 64, 4
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=61)
    _check(p, [300, 1, 0, 70, 129, 200, 64, 65], d, seed=62, memory=memory)


def test_varlen_layer_config4_style():
    """Config 4 at W = 2048: fixed-rate decays (the x-dependent decay input zeroed) with half-lives log-spaced
    2048 .. 1M tokens, the last KV head archival (never forgets), d = 5120, lengths across the window."""
    H, G, D, d, W, S = 24, 4, 256, 5120, 2048, 4
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=0, seed=63)
    life = torch.logspace(math.log10(2048), 6.0, G)
    p.ab_w[:G] = 0.0                                  # a = 0: g = -e^{A_log} softplus(dt_bias)
    p.ab_b[:G] = 0.0
    p.A_log = (math.log(2.0) / life / torch.nn.functional.softplus(p.dt_bias)).log()
    p.decay_mask = torch.ones(G)
    p.decay_mask[-1] = 0.0                            # the archival head is the last one
    _check(p, [2500, 700, 4100, 2049], d, seed=64)

"""The allocation-free decode step against the regular one, through the C ABI.

``bf_bifrost_layer_decode_noalloc`` exists for callers that cannot allocate device memory when they run a
decode step (a runtime whose memory manager already holds nearly all of HBM, or a host that binds only the
C entry points and cannot own a device workspace); it takes its scratch from a fixed array inside the
library instead of a caller workspace.  This test runs two decode steps in a row through both entry points
on identical copies of a cache and requires the same outputs and the same cache updates, with the memory on
and in the window-only mode (memory = 0).  The file name
makes pytest collect it last, so a run that stops at the first failure has run every other test already.
"""
import ctypes

import pytest
import torch

from oracle import bifrost_oracle as ob
from params import layer_params

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("memory", [1, 0])
def test_noalloc_decode_matches_workspace_decode(memory):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda")
    from heimdall_b200 import BifrostLayer, _lib
    from heimdall_b200.functional import ptr
    from heimdall_b200.structs import BfRingCache

    H, G, D, d, W, S, B = 24, 4, 256, 128, 64, 4, 3
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=21)
    L = BifrostLayer.from_params(p, dev)
    gen = torch.Generator(device=dev).manual_seed(4)
    r = lambda *s: torch.randn(*s, generator=gen, device=dev)
    bf = torch.bfloat16
    rms = lambda z: z * torch.rsqrt(z.square().mean(-1, keepdim=True) + 1e-6)
    pos = torch.tensor([700, 1000, 5000], device=dev, dtype=torch.int64)
    rp_abs = pos[:, None] - W + torch.arange(W, device=dev)[None]
    ring_pos = torch.empty(B, W, dtype=torch.int64, device=dev).scatter_(1, rp_abs % W, rp_abs)
    base = dict(ring_k=rms(r(B, G, W, D)).to(bf), ring_v=rms(r(B, G, W, D)).to(bf),
                ring_km=torch.nn.functional.normalize(r(B, W, G, D), dim=-1),
                ring_g=-torch.rand(B, W, G, generator=gen, device=dev) * 0.05,
                ring_beta=torch.rand(B, W, G, generator=gen, device=dev), ring_pos=ring_pos,
                sink_k=rms(r(B, G, S, D)).to(bf), sink_v=rms(r(B, G, S, D)).to(bf), S=r(B, G, D, D) * 0.05)
    caches = [{k: v.clone() for k, v in base.items()} for _ in range(2)]
    structs = [BfRingCache(ptr(c["ring_k"]), ptr(c["ring_v"]), ptr(c["ring_km"]), ptr(c["ring_g"]),
                           ptr(c["ring_beta"]), ptr(c["ring_pos"]), W, ptr(c["sink_k"]), ptr(c["sink_v"]), S,
                           ptr(c["S"])) for c in caches]
    nws = _lib.size("bf_layer_decode_workspace", B, H, G, D, W)
    ws = torch.empty(nws, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    lay = ctypes.addressof(L.struct)
    for step in range(2):   # two calls in a row: the shared scratch keeps the first call's contents
        x, q, k, v = r(B, d).to(bf), rms(r(B, H, D)).to(bf), rms(r(B, G, D)).to(bf), rms(r(B, G, D)).to(bf)
        qr, kr = rms(r(B, H, D)).to(bf), rms(r(B, G, D)).to(bf)
        o_ref = torch.empty(B, H, D, device=dev)
        o_new = torch.full((B, H, D), float("nan"), device=dev)
        lse_ref = torch.empty(B, H, device=dev)
        lse_new = torch.empty(B, H, device=dev)
        _lib.call("bf_bifrost_layer_decode", lay, ptr(x), ptr(q), ptr(k), ptr(v), ptr(qr), ptr(kr), ptr(pos), B,
                  ctypes.addressof(structs[0]), memory, ptr(o_ref), ptr(lse_ref), ptr(ws), nws, stream)
        _lib.call("bf_bifrost_layer_decode_noalloc", lay, ptr(x), ptr(q), ptr(k), ptr(v), ptr(qr), ptr(kr), ptr(pos),
                  B, ctypes.addressof(structs[1]), memory, ptr(o_new), ptr(lse_new), stream)
        torch.cuda.synchronize()
        assert ob.rel_l2(o_new.cpu(), o_ref.cpu()) < 1e-6, step
        assert ob.rel_l2(lse_new.cpu(), lse_ref.cpu()) < 1e-6, step
        for key in base:
            assert ob.rel_l2(caches[1][key].cpu().double(), caches[0][key].cpu().double()) < 1e-6, (step, key)
        pos += 1
    # a batch that does not fit the fixed scratch is refused before anything runs
    with pytest.raises(_lib.BifrostError) as e:
        _lib.call("bf_bifrost_layer_decode_noalloc", lay, ptr(x), ptr(q), ptr(k), ptr(v), ptr(qr), ptr(kr), ptr(pos),
                  4096, ctypes.addressof(structs[1]), 1, ptr(o_new), ptr(lse_new), stream)
    assert e.value.code == 4

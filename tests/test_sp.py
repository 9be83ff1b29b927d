"""Sequence-parallel layer prefill (heimdall_b200.sp) on CPU: two gloo ranks run the real orchestration --
sinks broadcast, halo exchange, write stream, segment maps, all-gather, prefix fold, halo cache -- with the
oracle standing in for the GPU kernels (a test-side engine: a layer object with the BifrostLayer methods,
and the two segment functions patched), and the concatenated outputs must equal the oracle's one pass
over the whole sequence (the mixed-parts property of the reference, tests/test_hibrit.py:78-90)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import bifrost_oracle as ob
from params import layer_params

H, G, D, DM, W, S, T = 4, 2, 32, 16, 8, 2, 20   # T tokens per rank


class OracleLayer:
    """The BifrostLayer methods student_sp calls, computed by the CPU oracle."""

    def __init__(self, p):
        self.p, self.window, self.sinks = p, p.window, p.sinks

    def mem_inputs(self, x, q, k, pos0=0, pos=None):
        t = x.shape[1]
        qm, km, g, beta = ob.mem_inputs(self.p, x.double(), q.double(), k.double(), torch.arange(pos0, pos0 + t),
                                        dtype=torch.float64)
        return qm.float(), km.float(), g.float(), beta.float(), None   # the GPU layer's output dtypes

    def student(self, x, q, k, v, qr, kr, start, cache=None, memory=True):
        return ob.student(self.p, x.double(), q.double(), k.double(), v.double(), qr.double(), kr.double(), start,
                          cache, memory=memory, dtype=torch.float64)

    def prefill_sp_begin(self, x, q, k, v, qr, kr, start, cache):
        from heimdall_b200 import sp
        t, W = x.shape[1], self.window
        _, km, g, beta, _ = self.mem_inputs(x, q, k, pos0=start)
        if start == 0:
            kw, gw, bw, vw = sp.write_stream(None, None, None, None, km, g, beta, v, t, W, True)
        else:   # the halo in time order, read back from the ring (slot = position mod W)
            idx = torch.arange(start - W, start) % W
            kw, gw, bw, vw = sp.write_stream(cache["ring_km"][:, idx], cache["ring_g"][:, idx],
                                             cache["ring_beta"][:, idx], cache["ring_v"][:, :, idx].transpose(1, 2),
                                             km, g, beta, v, t, W, False)
        M, N = oracle_segment_transform(kw, vw, gw, bw)
        return M, N, (x, q, k, v, qr, kr, start, cache)

    def prefill_sp_finish(self, h):
        x, q, k, v, qr, kr, start, cache = h
        return self.student(x, q, k, v, qr, kr, start, cache, True)


def oracle_segment_transform(k, v, g, beta, s0=None):
    B, n, Gh, Dd = k.shape
    eye = torch.eye(Dd, dtype=torch.float64).expand(B, Gh, Dd, Dd).contiguous()
    kk, vv, gg, bb = k.double(), v.double(), g.double(), beta.double()
    _, M = ob.gdn_chunked(kk, kk, torch.zeros_like(vv), gg, bb, 8, eye, dtype=torch.float64)
    _, N = ob.gdn_chunked(kk, kk, vv, gg, bb, 8, None, dtype=torch.float64)
    return M.float(), N.float()


def oracle_apply_prefix(M, N, s0=None):
    n = M.shape[0]
    out = [torch.zeros_like(M[0]) if s0 is None else s0.double()] if n else [torch.zeros(M.shape[1:], dtype=M.dtype)]
    for j in range(n):
        out.append(M[j].double() @ out[-1].double() + N[j].double())
    return torch.stack(out).float()


def _inputs(seed=3):
    gen = torch.Generator().manual_seed(seed)
    rms = lambda z: z * torch.rsqrt(z.square().mean(-1, keepdim=True) + 1e-6)
    bf = lambda z: z.to(torch.bfloat16)
    n = 2 * T
    return (bf(torch.randn(1, n, DM, generator=gen)), bf(rms(torch.randn(1, n, H, D, generator=gen))),
            bf(rms(torch.randn(1, n, G, D, generator=gen))), bf(rms(torch.randn(1, n, G, D, generator=gen))),
            bf(rms(torch.randn(1, H, n, D, generator=gen))), bf(rms(torch.randn(1, G, n, D, generator=gen))))


def _rank_main(rank, world, port, memory, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from heimdall_b200 import sp
        sp.F_.apply_prefix = oracle_apply_prefix
        p = layer_params(H, G, D, DM, window=W, sinks=S, archival=1, seed=5)
        x, q, k, v, qr, kr = _inputs()
        sl = slice(rank * T, (rank + 1) * T)
        o, cache = sp.student_sp(OracleLayer(p), x[:, sl], q[:, sl], k[:, sl], v[:, sl], qr[:, :, sl],
                                 kr[:, :, sl], memory=memory)
        torch.save({"o": o, "S": cache.get("S")}, f"{out_path}.{rank}")
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("memory", [True, False])
def test_sp_two_ranks_equals_one_pass(tmp_path, memory):
    out = str(tmp_path / "sp")
    mp.spawn(_rank_main, args=(2, _free_port(), memory, out), nprocs=2, join=True)
    p = layer_params(H, G, D, DM, window=W, sinks=S, archival=1, seed=5)
    x, q, k, v, qr, kr = _inputs()
    cache = {}
    o_ref = ob.student(p, *(z.double() for z in (x, q, k, v, qr, kr)), 0, cache, memory=memory,
                       dtype=torch.float64)
    parts = [torch.load(f"{out}.{r}") for r in range(2)]
    o = torch.cat([pt["o"] for pt in parts], 1)
    # equal up to the fp32 rounding of the cache entries handed across the segment boundary
    assert ob.rel_l2(o, o_ref) < 1e-5
    if memory:   # the incoming state of rank 1 + its own segment == the one-pass state (in its cache)
        assert ob.rel_l2(parts[1]["S"], cache["S"]) < 1e-5


def test_write_stream_and_halo_cache_layout():
    from heimdall_b200 import sp
    B, n = 1, 12
    km = torch.arange(n * 2.0).reshape(1, n, 2, 1)
    g = torch.arange(n * 2.0).reshape(1, n, 2)
    beta = g + 100
    v = km + 200
    h = [z[:, -4:] for z in (km, g, beta, v)]
    own = sp.write_stream(*h, km, g, beta, v, T=n, W=4, first=False)
    assert own[0].shape[1] == n and torch.equal(own[0][:, :4], h[0]) and torch.equal(own[0][:, 4:], km[:, :n - 4])
    first = sp.write_stream(None, None, None, None, km, g, beta, v, T=n, W=4, first=True)
    assert first[0].shape[1] == n - 4
    kr_h = torch.arange(4.0).reshape(1, 1, 4, 1)
    c = sp.halo_cache(kr_h, v[:, -4:, :1], km[:, -4:, :1], g[:, -4:, :1], beta[:, -4:, :1], None, None, None,
                      start=10, W=4)
    # positions 6..9 land in slots 2, 3, 0, 1
    assert c["ring_pos"].tolist() == [8, 9, 6, 7]
    assert c["ring_k"].flatten().tolist() == [2.0, 3.0, 0.0, 1.0]

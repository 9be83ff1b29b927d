"""Sequence-parallel pieces on the GPU: the segment state map against the oracle (and its defining property
S_out = M S_in + N), the prefix fold against fp64, the whole decomposition emulated on one GPU, and
student_sp on two GPUs (NCCL) against one pass on one GPU."""
import os
import socket

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


def _stream(B, T, G, D, seed):
    gen = torch.Generator().manual_seed(seed)
    k = F.normalize(torch.randn(B, T, G, D, generator=gen), dim=-1)
    v = torch.randn(B, T, G, D, generator=gen).to(torch.bfloat16)
    g = -torch.rand(B, T, G, generator=gen) * 0.02   # half-lives of 35 tokens and more
    beta = torch.rand(B, T, G, generator=gen)
    return k, v, g, beta


@pytest.mark.parametrize("T", [1, 128, 300, 2000])
def test_segment_transform_matches_oracle(T):
    dev = _dev()
    from heimdall_b200.functional import delta_rule_gqa, segment_transform
    B, G, D = 2, 4, 256
    k, v, g, beta = _stream(B, T, G, D, seed=T)
    M, N = segment_transform(*(z.to(dev) for z in (k, v, g, beta)))
    torch.cuda.synchronize()
    kk, vv = k.double(), v.double()
    eye = torch.eye(D, dtype=torch.float64).expand(B, G, D, D).contiguous()
    _, M_ref = ob.gdn_chunked(kk, kk, torch.zeros_like(vv), g.double(), beta.double(), 64, eye, dtype=torch.float64)
    _, N_ref = ob.gdn_chunked(kk, kk, vv, g.double(), beta.double(), 64, None, dtype=torch.float64)
    assert ob.rel_l2(M.cpu(), M_ref) < S_TOL and ob.rel_l2(N.cpu(), N_ref) < S_TOL
    # defining property: from any incoming state the segment ends at M S + N
    S_in = torch.randn(B, G, D, D, generator=torch.Generator().manual_seed(1)) * 0.05
    q = torch.zeros(B, T, G, 1, D)
    _, S_out = delta_rule_gqa(q.to(dev), k.to(dev), v.to(dev), g.to(dev), beta.to(dev), 64, S_in.to(dev))
    torch.cuda.synchronize()
    assert ob.rel_l2(S_out.cpu(), M.cpu() @ S_in + N.cpu()) < S_TOL


def test_apply_prefix_matches_fp64():
    dev = _dev()
    from heimdall_b200.functional import apply_prefix
    n, B, G, D = 5, 2, 4, 256
    gen = torch.Generator().manual_seed(2)
    M = torch.eye(D).expand(n, B, G, D, D) * 0.9 + torch.randn(n, B, G, D, D, generator=gen) * 0.01
    N = torch.randn(n, B, G, D, D, generator=gen) * 0.1
    s0 = torch.randn(B, G, D, D, generator=gen) * 0.1
    S = apply_prefix(M.to(dev), N.to(dev), s0.to(dev))
    torch.cuda.synchronize()
    ref = [s0.double()]
    for j in range(n):
        ref.append(M[j].double() @ ref[-1] + N[j].double())
    assert ob.rel_l2(S.cpu(), torch.stack(ref)) < 1e-5
    S0 = apply_prefix(M[:0].to(dev), N[:0].to(dev))
    assert S0.shape[0] == 1 and float(S0.abs().max()) == 0.0


def _layer_inputs(H, G, D, d, T, seed, B=1):
    gen = torch.Generator().manual_seed(seed)
    rms = lambda z: z * torch.rsqrt(z.square().mean(-1, keepdim=True) + 1e-6)
    bf = lambda z: z.to(torch.bfloat16)
    return (bf(torch.randn(B, T, d, generator=gen)), bf(rms(torch.randn(B, T, H, D, generator=gen))),
            bf(rms(torch.randn(B, T, G, D, generator=gen))), bf(rms(torch.randn(B, T, G, D, generator=gen))),
            bf(rms(torch.randn(B, H, T, D, generator=gen))), bf(rms(torch.randn(B, G, T, D, generator=gen))))


def test_sp_decomposition_emulated_on_one_gpu():
    """The ranks of student_sp run one after another on one GPU (no collectives): halo, write stream,
    segment maps, prefix fold and halo caches give the one-pass outputs and final state."""
    dev = _dev()
    from heimdall_b200 import BifrostLayer, sp
    from heimdall_b200.functional import apply_prefix, segment_transform
    H, G, D, d, W, S, P, T = 24, 4, 256, 128, 256, 4, 3, 640
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=4)
    L = BifrostLayer.from_params(p, dev)
    ins = [z.to(dev) for z in _layer_inputs(H, G, D, d, P * T, seed=6)]
    x, q, k, v, qr, kr = ins
    cache_1 = {}
    o_1 = L.student(x, q, k, v, qr, kr, 0, cache_1)
    parts = []
    for j in range(P):
        sl = slice(j * T, (j + 1) * T)
        xs, qs, ks, vs, qrs, krs = (x[:, sl], q[:, sl], k[:, sl], v[:, sl], qr[:, :, sl].contiguous(),
                                    kr[:, :, sl].contiguous())
        parts.append((xs.contiguous(), qs.contiguous(), ks.contiguous(), vs.contiguous(), qrs, krs))
    Ms, Ns, halos = [], [], [None]
    for j in range(P):
        xs, qs, ks, vs, qrs, krs = parts[j]
        _, km, g, beta, _ = L.mem_inputs(xs, qs, ks, pos0=j * T)
        if j == 0:
            kw, gw, bw, vw = sp.write_stream(None, None, None, None, km, g, beta, vs, T, W, True)
        else:
            px, _, pk, pv, _, pkr = parts[j - 1]
            halo = [px[:, -W:].contiguous(), pk[:, -W:].contiguous(), pv[:, -W:].contiguous(),
                    pkr[:, :, -W:].contiguous()]
            km_h, g_h, b_h = sp._halo_inputs(L, halo, j * T, W, qs)
            halos.append((halo, km_h, g_h, b_h))
            kw, gw, bw, vw = sp.write_stream(km_h, g_h, b_h, halo[2], km, g, beta, vs, T, W, False)
        M, N = segment_transform(kw, vw, gw, bw)
        Ms.append(M)
        Ns.append(N)
    S_all = apply_prefix(torch.stack(Ms), torch.stack(Ns))
    sink_k = parts[0][5][:, :, :S].contiguous()
    sink_v = parts[0][3][:, :S].transpose(1, 2).contiguous()
    outs = []
    for j in range(P):
        if j == 0:
            cache = {"S": S_all[0].contiguous()}
        else:
            halo, km_h, g_h, b_h = halos[j]
            cache = sp.halo_cache(halo[3], halo[2], km_h, g_h, b_h, sink_k, sink_v, S_all[j].contiguous(), j * T, W)
        outs.append(L.student(*parts[j], j * T, cache))
    torch.cuda.synchronize()
    assert ob.rel_l2(torch.cat(outs, 1).cpu(), o_1.cpu()) < O_TOL
    assert ob.rel_l2(cache["S"].cpu(), cache_1["S"].cpu()) < S_TOL
    assert ob.rel_l2(S_all[P].cpu(), cache_1["S"].cpu()) < S_TOL


def _sp_rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from heimdall_b200 import BifrostLayer, sp
        H, G, D, d, W, S, T = 24, 4, 256, 128, 256, 4, 512
        p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=8)
        L = BifrostLayer.from_params(p, dev)
        x, q, k, v, qr, kr = _layer_inputs(H, G, D, d, world * T, seed=9)
        sl = slice(rank * T, (rank + 1) * T)
        o, cache = sp.student_sp(L, *(z.to(dev) for z in (x[:, sl], q[:, sl], k[:, sl], v[:, sl], qr[:, :, sl],
                                                            kr[:, :, sl])))
        torch.cuda.synchronize()
        torch.save({"o": o.cpu(), "S": cache["S"].cpu()}, f"{out}.{rank}")
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_student_sp_two_gpus(tmp_path):
    dev = _dev()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    out = str(tmp_path / "sp")
    mp.spawn(_sp_rank, args=(2, port, out), nprocs=2, join=True)
    from heimdall_b200 import BifrostLayer
    H, G, D, d, W, S, T = 24, 4, 256, 128, 256, 4, 512
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=8)
    L = BifrostLayer.from_params(p, dev)
    x, q, k, v, qr, kr = (z.to(dev) for z in _layer_inputs(H, G, D, d, 2 * T, seed=9))
    cache = {}
    o_ref = L.student(x, q, k, v, qr, kr, 0, cache)
    torch.cuda.synchronize()
    parts = [torch.load(f"{out}.{r}") for r in range(2)]
    assert ob.rel_l2(torch.cat([pt["o"] for pt in parts], 1), o_ref.cpu()) < O_TOL
    assert ob.rel_l2(parts[1]["S"], cache["S"].cpu()) < S_TOL


def _sp_graph_rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    gr = None
    try:
        from heimdall_b200 import BifrostLayer, sp
        H, G, D, d, W, S, T = 24, 4, 256, 128, 256, 4, 512
        p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=8)
        L = BifrostLayer.from_params(p, dev)
        sl = slice(rank * T, (rank + 1) * T)
        part = lambda seed: [z.to(dev, torch.bfloat16).contiguous() for z in (lambda a: (
            a[0][:, sl], a[1][:, sl], a[2][:, sl], a[3][:, sl], a[4][:, :, sl], a[5][:, :, sl]))(
            _layer_inputs(H, G, D, d, world * T, seed=seed))]
        a, b = part(9), part(10)
        gr = sp.StudentSPGraph(L, *[z.clone() for z in a])
        res = {}
        for name, ins in (("a", a), ("b", b), ("a2", a)):      # new tokens copied into the graph's inputs
            for dst, src in zip(gr.inputs, ins):
                dst.copy_(src)
            gr.replay()
            gr.check()
            torch.cuda.synchronize()
            res[name] = {"o": gr.o.cpu(), "S": gr.cache["S"].cpu()}
        o_e, c_e = sp.student_sp(L, *b)
        torch.cuda.synchronize()
        res["eager_b"] = {"o": o_e.cpu(), "S": c_e["S"].cpu()}
        torch.save(res, f"{out}.{rank}")
        dist.barrier()
    finally:
        gr = None                 # the graph holds NCCL calls: release it before the process group
        torch.cuda.synchronize()
        dist.destroy_process_group()


def test_student_sp_graph_two_gpus(tmp_path):
    """The captured step (StudentSPGraph) replayed with two sets of tokens equals the eager step and one
    prefill of the whole sequence on one GPU."""
    dev = _dev()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    out = str(tmp_path / "spg")
    mp.spawn(_sp_graph_rank, args=(2, port, out), nprocs=2, join=True)
    from heimdall_b200 import BifrostLayer
    H, G, D, d, W, S, T = 24, 4, 256, 128, 256, 4, 512
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=8)
    L = BifrostLayer.from_params(p, dev)
    parts = [torch.load(f"{out}.{r}") for r in range(2)]
    for seed, name in ((9, "a"), (10, "b"), (9, "a2")):
        x, q, k, v, qr, kr = (z.to(dev) for z in _layer_inputs(H, G, D, d, 2 * T, seed=seed))
        cache = {}
        o_ref = L.student(x, q, k, v, qr, kr, 0, cache)
        torch.cuda.synchronize()
        assert ob.rel_l2(torch.cat([pt[name]["o"] for pt in parts], 1), o_ref.cpu()) < O_TOL, name
        assert ob.rel_l2(parts[1][name]["S"], cache["S"].cpu()) < S_TOL, name
    for r in range(2):
        assert ob.rel_l2(parts[r]["b"]["o"], parts[r]["eager_b"]["o"]) < 1e-5
        assert ob.rel_l2(parts[r]["b"]["S"], parts[r]["eager_b"]["S"]) < 1e-5


def _cache_cpu(c):
    return {k_: (v_.cpu().float() if v_.is_floating_point() else v_.cpu()) for k_, v_ in c.items()}


def test_two_phase_prefill_matches_one_call():
    """prefill_sp_begin + prefill_sp_finish (the second phase turns the map pass's per-chunk states into the
    states from the incoming state with the fix-up, no second scan) against the oracle's prefill from the same
    cache and against one GPU prefill; the begin phase's state map equals segment_transform of the segment's
    write stream (halo tokens, then this rank's tokens)."""
    dev = _dev()
    from heimdall_b200 import BifrostLayer, sp
    from heimdall_b200.functional import segment_transform
    H, G, D, d, W, S, T = 24, 4, 256, 128, 256, 4, 700
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=12)
    L = BifrostLayer.from_params(p, dev)
    x, q, k, v, qr, kr = (z.to(dev) for z in _layer_inputs(H, G, D, d, 2 * T, seed=13))
    start = T
    prev = (x[:, :T], k[:, :T], v[:, :T], kr[:, :, :T])
    halo = [prev[0][:, -W:].contiguous(), prev[1][:, -W:].contiguous(), prev[2][:, -W:].contiguous(),
            prev[3][:, :, -W:].contiguous()]
    mine = [x[:, T:].contiguous(), q[:, T:].contiguous(), k[:, T:].contiguous(), v[:, T:].contiguous(),
            qr[:, :, T:].contiguous(), kr[:, :, T:].contiguous()]
    km_h, g_h, b_h = sp._halo_inputs(L, halo, start, W, mine[1])
    sink_k, sink_v = kr[:, :, :S].contiguous(), v[:, :S].transpose(1, 2).contiguous()
    S_in = torch.randn(1, G, D, D, generator=torch.Generator().manual_seed(3)).to(dev) * 0.05
    c1 = sp.halo_cache(halo[3], halo[2], km_h, g_h, b_h, sink_k, sink_v, S_in.clone(), start, W)
    c_ref = _cache_cpu(c1)
    o1 = L.student(*mine, start, c1)
    c2 = sp.halo_cache(halo[3], halo[2], km_h, g_h, b_h, sink_k, sink_v, None, start, W)
    M, N, h = L.prefill_sp_begin(*mine, start, c2)
    c2["S"].copy_(S_in)
    o2 = L.prefill_sp_finish(h)
    torch.cuda.synchronize()
    o_ref = ob.student(p, *(z.cpu().float() for z in mine), start, c_ref)
    assert ob.rel_l2(o2.cpu(), o_ref) < O_TOL
    assert ob.rel_l2(c2["S"].cpu(), c_ref["S"]) < S_TOL
    assert ob.rel_l2(o2.cpu(), o1.cpu()) < O_TOL
    assert ob.rel_l2(c2["S"].cpu(), c1["S"].cpu()) < S_TOL
    _, km, g, beta, _ = L.mem_inputs(mine[0], mine[1], mine[2], pos0=start)
    kw, gw, bw, vw = sp.write_stream(km_h, g_h, b_h, halo[2], km, g, beta, mine[3], T, W, False)
    M2, N2 = segment_transform(kw, vw, gw, bw)
    torch.cuda.synchronize()
    assert ob.rel_l2(M.cpu(), M2.cpu()) < 1e-5 and ob.rel_l2(N.cpu(), N2.cpu()) < 1e-5


def test_abandoned_first_phase_is_safe():
    """A first phase whose handle is dropped without the second phase: its window kernel (still running on a
    side stream when prefill_sp_begin returns) is waited for before the handle's buffers are released, so a
    prefill that reuses the memory right after is unaffected."""
    import gc
    dev = _dev()
    from heimdall_b200 import BifrostLayer, sp
    H, G, D, d, W, S, T = 24, 4, 256, 128, 256, 4, 700
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=12)
    L = BifrostLayer.from_params(p, dev)
    x, q, k, v, qr, kr = (z.to(dev) for z in _layer_inputs(H, G, D, d, 2 * T, seed=13))
    start = T
    halo = [x[:, T - W:T].contiguous(), k[:, T - W:T].contiguous(), v[:, T - W:T].contiguous(),
            kr[:, :, T - W:T].contiguous()]
    mine = [x[:, T:].contiguous(), q[:, T:].contiguous(), k[:, T:].contiguous(), v[:, T:].contiguous(),
            qr[:, :, T:].contiguous(), kr[:, :, T:].contiguous()]
    km_h, g_h, b_h = sp._halo_inputs(L, halo, start, W, mine[1])
    sink_k, sink_v = kr[:, :, :S].contiguous(), v[:, :S].transpose(1, 2).contiguous()
    S_in = torch.randn(1, G, D, D, generator=torch.Generator().manual_seed(3)).to(dev) * 0.05
    c0 = sp.halo_cache(halo[3], halo[2], km_h, g_h, b_h, sink_k, sink_v, None, start, W)
    _, _, h = L.prefill_sp_begin(*mine, start, c0)
    del h
    gc.collect()
    c1 = sp.halo_cache(halo[3], halo[2], km_h, g_h, b_h, sink_k, sink_v, S_in.clone(), start, W)
    o1 = L.student(*mine, start, c1)
    c2 = sp.halo_cache(halo[3], halo[2], km_h, g_h, b_h, sink_k, sink_v, None, start, W)
    _, _, h2 = L.prefill_sp_begin(*mine, start, c2)
    c2["S"].copy_(S_in)
    o2 = L.prefill_sp_finish(h2)
    torch.cuda.synchronize()
    assert ob.rel_l2(o2.cpu(), o1.cpu()) < O_TOL


def test_two_phase_fixup_production_geometry():
    """The fix-up at the production geometry (W = 2048, d = 5120): the second of two 8192-token segments runs
    the two-phase prefill from the first segment's real final state (its transitions over 64 chunks, with an
    archival head that never decays), against one prefill of all 16384 tokens."""
    dev = _dev()
    from heimdall_b200 import BifrostLayer, sp
    H, G, D, d, W, S, T = 24, 4, 256, 5120, 2048, 4, 8192
    p = layer_params(H, G, D, d, window=W, sinks=S, archival=1, seed=15)
    L = BifrostLayer.from_params(p, dev)
    x, q, k, v, qr, kr = (z.to(dev) for z in _layer_inputs(H, G, D, d, 2 * T, seed=16))
    cache_1 = {}
    o_1 = L.student(x, q, k, v, qr, kr, 0, cache_1)
    part = lambda z, a, b: z[:, a:b].contiguous()
    partT = lambda z, a, b: z[:, :, a:b].contiguous()
    cache_a = {}
    L.student(part(x, 0, T), part(q, 0, T), part(k, 0, T), part(v, 0, T), partT(qr, 0, T), partT(kr, 0, T), 0, cache_a)
    mine = [part(x, T, 2 * T), part(q, T, 2 * T), part(k, T, 2 * T), part(v, T, 2 * T), partT(qr, T, 2 * T),
            partT(kr, T, 2 * T)]
    halo = [part(x, T - W, T), part(k, T - W, T), part(v, T - W, T), partT(kr, T - W, T)]
    km_h, g_h, b_h = sp._halo_inputs(L, halo, T, W, mine[1])
    c = sp.halo_cache(halo[3], halo[2], km_h, g_h, b_h, kr[:, :, :S].contiguous(), v[:, :S].transpose(1, 2).contiguous(),
                      None, T, W)
    M, N, h = L.prefill_sp_begin(*mine, T, c)
    c["S"].copy_(cache_a["S"])
    o_b = L.prefill_sp_finish(h)
    torch.cuda.synchronize()
    assert ob.rel_l2(o_b.cpu(), o_1[:, T:].cpu()) < O_TOL
    assert ob.rel_l2(c["S"].cpu(), cache_1["S"].cpu()) < S_TOL
    # the segment map itself: S_out = M S_in + N reproduces the one-pass state
    assert ob.rel_l2((M @ cache_a["S"] + N).cpu(), cache_1["S"].cpu()) < S_TOL

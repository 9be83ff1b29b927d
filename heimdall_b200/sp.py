"""Sequence-parallel prefill of one Bifrost layer: a long sequence split into consecutive segments, one per
rank (one GPU per rank, ``torch.distributed`` over NCCL).

The layer is ``HybridAttention._student`` (heimdall/hibrit.py:363-424) run over the whole sequence from an
empty cache.  Rank j holds tokens [j T, (j+1) T) and returns their outputs.  Two things cross segments:

* the window: a token sees the previous W tokens and the S sinks, so rank j needs the last W tokens of
  rank j-1 (a halo: x, k, v, kr) and the first S tokens of rank 0;
* the memory: the delta-rule state after all earlier tokens.  Memory writes lag the window by W
  (hibrit.py:391-396), so rank j's write stream is the W halo tokens followed by its first T - W tokens.
  Each rank computes the state map of its write stream, (M_j, N_j) with S_out = M_j S_in + N_j, the maps
  are all-gathered, and each rank folds the earlier ones into its incoming state
  (``functional.apply_prefix``).

Rank j runs the layer prefill of its tokens from a cache built from the halo: the ring holds the halo
tokens (slot = position mod W), the sinks are rank 0's first tokens and S is the incoming state.  A
prefill from such a cache is exactly the continuation of the sequence (the reference's mixed-parts
property, tests/test_hibrit.py:78-90), so the outputs equal one pass over the whole sequence.  The
prefill runs in two phases on one workspace (``BifrostLayer.prefill_sp_begin`` / ``prefill_sp_finish``):
the first computes the memory inputs, the per-chunk products and the state map, the second everything
that depends on the incoming state, so nothing is computed twice.  The window attention depends on no state:
the first phase launches it on a low-priority side stream and returns while it runs, so that it fills the SMs
the two sequential scans leave free; the second phase joins it before the memory reads.  The rest of the call
runs on a high-priority stream, and the exchange should run on a high-priority NCCL stream too (a process group made with
``ProcessGroupNCCL.Options(is_high_priority_stream=True)``), or its kernels wait behind the window's CTAs.

Traffic per rank and layer: the halo (W tokens of x, k, v, kr: 33 MB at W = 2048, d = 5120) from the left
neighbour, the sink rows from rank 0, and an all-gather of (M, N) (2 MB per rank at G = 4, D = 256).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import functional as F_


def _peer(group, r: int) -> int:
    return dist.get_global_rank(group, r) if group is not None else r


def _p2p_shift(tensors, rank: int, world: int, group):
    """Send ``tensors`` to rank+1 and receive the same shapes from rank-1 (None on rank 0), as one batch
    of point-to-point operations."""
    ops, recv = [], None
    send = [t.contiguous() for t in tensors]          # held until the sends completed
    if rank > 0:
        recv = [torch.empty_like(t) for t in send]
        ops += [dist.P2POp(dist.irecv, r, _peer(group, rank - 1), group) for r in recv]
    if rank < world - 1:
        ops += [dist.P2POp(dist.isend, t, _peer(group, rank + 1), group) for t in send]
    if ops:
        for r in dist.batch_isend_irecv(ops):
            r.wait()
    return recv


def write_stream(km_h, g_h, b_h, v_h, km, g, beta, v, T: int, W: int, first: bool):
    """The segment's memory write stream: write step u uses the token W positions back, i.e. halo token u
    for u < W, then this rank's token u - W.  Rank 0 has no halo and T - W steps."""
    n_own = max(0, T - W)
    own = (km[:, :n_own], g[:, :n_own], beta[:, :n_own], v[:, :n_own])
    if first:
        return own
    return tuple(torch.cat((h, o), 1) for h, o in zip((km_h, g_h, b_h, v_h), own))


def halo_cache(kr_h, v_h, km_h, g_h, b_h, sink_k, sink_v, S_in, start: int, W: int):
    """The reference cache (hibrit.py:414-423) a rank starts from: ring = the W tokens before ``start`` in
    slot order (slot = position mod W), the sinks, and the incoming state."""
    dev = kr_h.device
    pos = torch.arange(start - W, start, device=dev, dtype=torch.int64)
    slot = pos % W
    B, G, _, D = kr_h.shape
    ring_k = torch.empty_like(kr_h)
    ring_k[:, :, slot] = kr_h
    ring_v = torch.empty(B, G, W, D, device=dev, dtype=v_h.dtype)
    ring_v[:, :, slot] = v_h.transpose(1, 2)
    ring_km = torch.empty_like(km_h)
    ring_km[:, slot] = km_h
    ring_g = torch.empty_like(g_h)
    ring_g[:, slot] = g_h
    ring_beta = torch.empty_like(b_h)
    ring_beta[:, slot] = b_h
    ring_pos = torch.empty(W, device=dev, dtype=torch.int64)
    ring_pos[slot] = pos
    cache = dict(ring_k=ring_k, ring_v=ring_v, ring_km=ring_km, ring_g=ring_g, ring_beta=ring_beta,
                 ring_pos=ring_pos, sink_k=sink_k, sink_v=sink_v)
    if S_in is not None:
        cache["S"] = S_in
    return cache


def student_sp(L, x, q, k, v, qr, kr, group=None, memory: bool = True, timeline=None, phase_hook=None,
               validate: str = "deferred"):
    """One layer prefill of a sequence split over the ranks of ``group`` in rank order, from an empty cache.

    Every rank passes its own T consecutive tokens (the same T on every rank, T >= W) in the layouts of
    ``BifrostLayer.student``: x [B,T,d], q [B,T,H,D], k/v [B,T,G,D], qr [B,H,T,D], kr [B,G,T,D] (bf16, on
    this rank's GPU).  Returns (o, cache): this rank's outputs [B,T,H,D] fp32 and its cache after the call
    (on the last rank that is the cache of the whole sequence).  Every rank must call it (collectives).

    Every rank checks that the gathered state maps are finite (a rank that sent NaN or inf) and raises the same
    RuntimeError for a corrupted one.  ``validate``: "deferred" (default) checks on the device and raises at the
    start of the next call on this device, or at ``check_maps()``, so the host never waits for the exchange and
    keeps enqueueing ahead of the GPU; "sync" waits for the check and raises before returning; "off" skips it.
    (On CPU tensors the check is always immediate.)

    Instrumentation (optional, GPU only): ``timeline`` is a list that receives (label, CUDA event) pairs
    recorded on the call's stream at the start and after each step (halo exchanged, halo memory inputs, state
    map, maps gathered, incoming state folded, done); ``phase_hook(phase)`` is called right before each of the
    two layer phases (0: memory inputs, per-chunk products, state map and the window launch; 1: the rest), e.g.
    to install per-phase stage events with ``bf_stage_events``.
    """
    T = x.shape[1]
    if T < L.window or T < L.sinks:
        raise NotImplementedError("sequence parallelism needs at least one window (and the sinks) per rank")
    # The call runs on a high-priority stream: the window kernel, launched by the first phase on the
    # lowest-priority stream and left running, then yields the SMs to everything else of the call (the
    # exchange, the fold of the maps, the second scan) instead of holding them back until it ends.
    if validate not in ("deferred", "sync", "off"):
        raise ValueError("validate must be 'deferred', 'sync' or 'off'")
    if x.device.type != "cuda":   # the host logic on CPU tensors (a CPU restatement of the layer)
        o, cache, fin = _student_sp(L, x, q, k, v, qr, kr, group, memory, None, None)
        if fin is not None and validate != "off":
            _raise_if_corrupted((fin, None))
        return o, cache
    check_maps(x.device)          # the previous call's maps on this device
    cur = torch.cuda.current_stream(x.device)
    hp = _priority_stream(x.device)
    hp.wait_stream(cur)
    with torch.cuda.stream(hp):
        o, cache, fin = _student_sp(L, x, q, k, v, qr, kr, group, memory, timeline, phase_hook)
        finite = _flags_to_host(fin) if fin is not None and validate != "off" else None
    cur.wait_stream(hp)   # later work on the caller's stream (reuse of the inputs' memory included) waits
    for t in [o, *(z for z in cache.values() if isinstance(z, torch.Tensor))]:
        t.record_stream(cur)   # allocated on the priority stream, used on the caller's
    if finite is not None:
        if validate == "sync":
            _raise_if_corrupted(finite)
        elif validate == "deferred":
            _PENDING[torch.device(x.device).index] = finite
    return o, cache


_PENDING = {}   # device index -> (flags in pinned host memory, event) of the last call's gathered maps


class StudentSPGraph:
    """``student_sp`` captured once as a CUDA graph and replayed: the whole sequence-parallel step (sink
    broadcast, halo exchange, both layer phases with the window on its side stream, the all-gather of the
    state maps and the fold) is one graph launch per step.  The eager step issues about a hundred kernel,
    copy and NCCL calls from Python, and at 16K tokens per GPU that enqueue (about 2.5 ms) is longer than the
    GPU's work; the graph removes it.

    The graph reads fixed input buffers: ``inputs`` = (x, q, k, v, qr, kr) as given (bf16, contiguous; copy
    each step's tokens into them before ``replay()``).  ``o`` and ``cache`` are the graph's own tensors,
    rewritten by every replay (the same layouts as ``student_sp``'s results).  ``check()`` raises the
    corrupted-map error of the last replay (it waits for the device).  Every rank of ``group`` constructs it
    and replays it in step: the graph holds the collectives.  Construction runs ``warmup`` eager steps first
    (NCCL communicators, the point-to-point pairs included, side streams and kernel attributes are set up
    outside the capture)."""

    def __init__(self, L, x, q, k, v, qr, kr, group=None, memory: bool = True, warmup: int = 2):
        if x.device.type != "cuda":
            raise ValueError("StudentSPGraph needs CUDA tensors")
        bf = torch.bfloat16
        self.inputs = tuple(z if (z.dtype == bf and z.is_contiguous()) else z.to(bf).contiguous()
                            for z in (x, q, k, v, qr, kr))
        for _ in range(max(1, int(warmup))):
            student_sp(L, *self.inputs, group=group, memory=memory, validate="sync")
        torch.cuda.synchronize(x.device)
        self.graph = torch.cuda.CUDAGraph()
        hp = _priority_stream(x.device)
        with torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
            cur = torch.cuda.current_stream(x.device)
            hp.wait_stream(cur)
            with torch.cuda.stream(hp):
                self.o, self.cache, self._fin = _student_sp(L, *self.inputs, group, memory, None, None)
            cur.wait_stream(hp)
        torch.cuda.synchronize(x.device)

    def replay(self) -> None:
        """One step on the current stream."""
        self.graph.replay()

    def check(self) -> None:
        """Raise if a rank sent a non-finite state map in the last replay (waits for the device)."""
        if self._fin is not None:
            _raise_if_corrupted((self._fin.cpu(), None))


def check_maps(device=None) -> None:
    """Raise the RuntimeError of a corrupted state map received by the last ``student_sp`` call on ``device``
    (the current device when None) that deferred its check; waits for that check on the device if needed."""
    key = torch.device(device if device is not None else torch.cuda.current_device()).index
    if key is None:
        key = torch.cuda.current_device()
    pend = _PENDING.pop(key, None)
    if pend is not None:
        _raise_if_corrupted(pend)


_PRIORITY_STREAMS = {}


def _priority_stream(device):
    key = torch.device(device).index
    if key not in _PRIORITY_STREAMS:
        _PRIORITY_STREAMS[key] = torch.cuda.Stream(device=device, priority=-5)   # clamped to the greatest
    return _PRIORITY_STREAMS[key]


def _student_sp(L, x, q, k, v, qr, kr, group, memory, timeline, phase_hook):
    def mark(label):
        if timeline is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            timeline.append((label, ev))

    def hook(phase):
        if phase_hook is not None:
            phase_hook(phase)

    mark("start")
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    B, T = x.shape[:2]
    W, S = L.window, L.sinks
    start = rank * T
    bf = torch.bfloat16
    x, q, k, v, qr, kr = (z.to(bf).contiguous() for z in (x, q, k, v, qr, kr))
    # sinks: rank 0's first S tokens
    sink_k = kr[:, :, :S].contiguous()
    sink_v = v[:, :S].transpose(1, 2).contiguous()
    if world > 1 and S > 0:
        dist.broadcast(sink_k, src=_peer(group, 0), group=group)
        dist.broadcast(sink_v, src=_peer(group, 0), group=group)
    # halo: the last W tokens of the previous rank, and their memory inputs
    halo = _p2p_shift([x[:, -W:], k[:, -W:], v[:, -W:], kr[:, :, -W:]], rank, world, group)
    mark("halo_exchanged")
    first = rank == 0
    cache = {}
    if not first:
        km_h, g_h, b_h = _halo_inputs(L, halo, start, W, q)
        cache = halo_cache(halo[3], halo[2], km_h, g_h, b_h, sink_k, sink_v, None, start, W)
    mark("halo_inputs")
    if not memory:
        o = L.student(x, q, k, v, qr, kr, start, cache, memory=False)
        mark("done")
        return o, cache, None
    # phase 1: this segment's state map (memory inputs and per-chunk products are kept for phase 2)
    hook(0)
    M, N, handle = L.prefill_sp_begin(x, q, k, v, qr, kr, start, cache)
    mark("maps")
    if world > 1:
        Ml = [torch.empty_like(M) for _ in range(world)]
        Nl = [torch.empty_like(N) for _ in range(world)]
        dist.all_gather(Ml, M.contiguous(), group=group)
        dist.all_gather(Nl, N.contiguous(), group=group)
        Ms, Ns = torch.stack(Ml), torch.stack(Nl)
    else:
        Ms, Ns = M[None], N[None]
    mark("gathered")
    finite = _maps_finite(Ms, Ns)
    S_in = F_.apply_prefix(Ms[:rank], Ns[:rank])[rank]
    if cache.get("S") is not None:
        cache["S"].copy_(S_in)
    else:
        cache["S"] = S_in.contiguous()
    mark("folded")
    # phase 2: the rest of the layer from the incoming state
    hook(1)
    o = L.prefill_sp_finish(handle)
    mark("done")
    return o, cache, finite


def _maps_finite(Ms, Ns):
    """Per segment, whether its gathered state map is finite (a rank that sent NaN or inf), on the maps' device."""
    return torch.isfinite(Ms).flatten(1).all(1) & torch.isfinite(Ns).flatten(1).all(1)


def _flags_to_host(fin):
    """The flags copied to pinned host memory behind an event, so the check does not hold back the second
    phase: ``_raise_if_corrupted`` waits for the flags only, after it is launched."""
    host = torch.empty(fin.shape, dtype=torch.bool, pin_memory=True)
    host.copy_(fin, non_blocking=True)
    ev = torch.cuda.Event()
    ev.record()
    return host, ev


def _raise_if_corrupted(finite):
    """Every rank sees the same gathered maps, so every rank raises the same error for a corrupted one (the
    outputs and the cache of this call are then undefined)."""
    flags, ev = finite
    if ev is not None:
        ev.synchronize()
    bad = [j for j, ok in enumerate(flags.tolist()) if not ok]
    if bad:
        raise RuntimeError(f"sequence-parallel prefill: the state map of segment(s) {bad} is not finite "
                           f"(the rank(s) holding them sent corrupted maps)")


def _halo_inputs(L, halo, start: int, W: int, q):
    """Memory inputs (km, g, beta) of the halo tokens, at their positions start - W .. start - 1.
    Their query projections are not needed (those tokens' outputs belong to the previous rank)."""
    x_h, k_h = halo[0], halo[1]
    q_h = torch.zeros(q.shape[0], W, *q.shape[2:], device=q.device, dtype=q.dtype)
    _, km_h, g_h, b_h, _ = L.mem_inputs(x_h, q_h, k_h, pos0=start - W)
    return km_h, g_h, b_h

"""The converted Bifrost layer core on B200: the host mirror of ``HybridAttention._student``.

``BifrostLayer`` holds a converted layer's parameters on the device plus their tensor-core operand
layout, and ``BifrostLayer.student`` has the signature and cache-dict semantics of the reference's
``HybridAttention._student(x, q, k, v, qr, kr, start, cache, memory)`` (heimdall/hibrit.py:363-424):
the cache keeps the reference's keys and layouts (ring_k, ring_v, ring_km, ring_g, ring_beta, ring_pos,
sink_k, sink_v, S), so caches are interchangeable with the reference's and ``HybridLM.cache_bytes``
sees the same constant footprint.
"""
from __future__ import annotations

import weakref

import torch

from . import _lib
from .functional import check_cuda, ptr, stream_handle
from .structs import BfLayer, BfRingCache

PARAM_NAMES = ("fq", "fk", "ab_w", "ab_b", "mix_w", "mix_b", "mix_lse", "mem_scale", "A_log", "dt_bias",
               "decay_mask")


def _aligned_bytes(n: int, device, align: int = 1024) -> torch.Tensor:
    buf = torch.empty(n + align, dtype=torch.uint8, device=device)
    off = (-buf.data_ptr()) % align
    return buf[off:off + n]


class BifrostLayer:
    """A converted layer's parameters on one CUDA device.

    ``params`` maps the names in ``PARAM_NAMES`` to tensors (any device/dtype; stored fp32), shaped as
    HybridAttention.convert creates them (heimdall/hibrit.py:211-240): fq [H,D,D], fk [G,D,D],
    ab_w [2G,d], ab_b [2G], mix_w [H,d], mix_b [H], mix_lse [H], mem_scale [H], A_log [G], dt_bias [G],
    decay_mask [G].
    """

    def __init__(self, params: dict, window: int, sinks: int, device=None):
        device = torch.device(device or "cuda")
        if device.type != "cuda":
            raise RuntimeError("heimdall_b200 runs on CUDA only (there is no CPU fallback)")
        self.device = device
        self.p = {n: params[n].detach().to(device=device, dtype=torch.float32).contiguous() for n in PARAM_NAMES}
        self.window, self.sinks = int(window), int(sinks)
        self.H, D = self.p["fq"].shape[0], self.p["fq"].shape[-1]
        self.G, self.D, self.d = self.p["fk"].shape[0], D, self.p["ab_w"].shape[1]
        self.R = self.H // self.G
        nbytes = _lib.size("bf_layer_weights_bytes", self.H, self.G, self.D, self.d)
        self.wbuf = _aligned_bytes(nbytes, device)
        self._host_slots = None
        self.refresh()

    @classmethod
    def converted(cls, H: int, G: int, D: int, d: int, window: int, sinks: int, archival: int,
                  mem_init: str = "long", generator=None, device=None) -> "BifrostLayer":
        """Conversion-time parameters, as ``HybridAttention.convert`` creates them (heimdall/hibrit.py:211-240):
        fq/fk identities, ab/mix zero with mix bias -2, mix_lse 0, dt log-uniform in [1e-3, 1e-1] with
        dt_bias = softplus^-1(dt); "long": half-lives log-spaced from the window to 1e6 tokens and
        mem_scale = sqrt(D); "mamba": A in U[1, 16] and mem_scale 1.  The first ``archival`` KV heads never decay."""
        import math
        gen = generator
        dt = torch.exp(torch.empty(G).uniform_(math.log(1e-3), math.log(1e-1), generator=gen))
        if mem_init == "mamba":
            mem_scale = torch.ones(H)
            A_log = torch.empty(G).uniform_(1.0, 16.0, generator=gen).log()
        else:
            mem_scale = torch.full((H,), float(D) ** 0.5)
            life = torch.logspace(math.log10(max(window, 2)), 6.0, G)
            A_log = (math.log(2.0) / (life * dt)).log()
        mask = torch.ones(G)
        mask[:archival] = 0.0
        params = dict(fq=torch.eye(D).repeat(H, 1, 1), fk=torch.eye(D).repeat(G, 1, 1), ab_w=torch.zeros(2 * G, d),
                      ab_b=torch.zeros(2 * G), mix_w=torch.zeros(H, d), mix_b=torch.full((H,), -2.0),
                      mix_lse=torch.zeros(H), mem_scale=mem_scale, A_log=A_log,
                      dt_bias=dt + torch.log(-torch.expm1(-dt)), decay_mask=mask)
        return cls(params, window, sinks, device)

    @classmethod
    def from_module(cls, attn, device=None) -> "BifrostLayer":
        """From a converted reference ``HybridAttention`` (its new parameters and decay_mask buffer)."""
        params = dict(fq=attn.fq, fk=attn.fk, ab_w=attn.ab.weight, ab_b=attn.ab.bias, mix_w=attn.mix.weight,
                      mix_b=attn.mix.bias, mix_lse=attn.mix_lse, mem_scale=attn.mem_scale, A_log=attn.A_log,
                      dt_bias=attn.dt_bias, decay_mask=attn.decay_mask)
        return cls(params, attn.window, attn.sinks, device)

    @classmethod
    def from_params(cls, lp, device=None) -> "BifrostLayer":
        """From any object with the parameter attributes (e.g. the test oracle's ``LayerParams``)."""
        return cls({n: getattr(lp, n) for n in PARAM_NAMES}, lp.window, lp.sinks, device)

    def refresh(self) -> None:
        """Rebuild the operand layouts after the parameters changed."""
        p = self.p
        with torch.cuda.device(self.device):
            _lib.call("bf_prepare_layer_weights", ptr(p["fq"]), ptr(p["fk"]), ptr(p["ab_w"]), ptr(p["mix_w"]),
                      self.H, self.G, self.D, self.d, ptr(self.wbuf), self.wbuf.numel(), stream_handle())
        self._struct = BfLayer(ptr(self.wbuf), ptr(p["ab_b"]), ptr(p["mix_b"]), ptr(p["mix_lse"]),
                               ptr(p["mem_scale"]), ptr(p["A_log"]), ptr(p["dt_bias"]), ptr(p["decay_mask"]),
                               self.H, self.G, self.D, self.d, self.window, self.sinks)

    @property
    def struct(self) -> BfLayer:
        return self._struct

    # ------------------------------------------------------------------ memory inputs
    def mem_inputs(self, x, q, k, pos0: int = 0, pos=None):
        """qm, km, g, beta, mixx for tokens at positions pos0.. (mirror of _mem_inputs, hibrit.py:327-334).

        x [B,t,d], q [B,t,H,D], k [B,t,G,D] (bf16); returns qm [B,t,H,D], km [B,t,G,D], g, beta [B,t,G],
        mixx [B,t,H] (= mix(x), the input term of the gate), all fp32.
        """
        check_cuda(x, q, k)
        B, t = x.shape[:2]
        dev = x.device
        xb, qb, kb = (z.to(torch.bfloat16).contiguous() for z in (x, q, k))
        qm = torch.empty(B, t, self.H, self.D, device=dev, dtype=torch.float32)
        km = torch.empty(B, t, self.G, self.D, device=dev, dtype=torch.float32)
        g = torch.empty(B, t, self.G, device=dev, dtype=torch.float32)
        beta = torch.empty_like(g)
        mixx = torch.empty(B, t, self.H, device=dev, dtype=torch.float32)
        posp = None if pos is None else pos.to(device=dev, dtype=torch.int64).contiguous()
        _lib.call("bf_mem_inputs", ctypes_ref(self._struct), ptr(xb), ptr(qb), ptr(kb), ptr(posp), int(pos0), B, t,
                  ptr(qm), ptr(km), ptr(g), ptr(beta), ptr(mixx), stream_handle())
        return qm, km, g, beta, mixx

    # ------------------------------------------------------------------ the layer core
    def student(self, x, q, k, v, qr, kr, start: int, cache=None, memory: bool = True):
        """Mirror of ``HybridAttention._student`` (heimdall/hibrit.py:363-424); returns o [B,t,H,D] fp32."""
        check_cuda(x, q, k, v, qr, kr)
        t = x.shape[1]
        if cache is not None and t == 1 and "ring_k" in cache:
            return self._decode(x, q, k, v, qr, kr, int(start), cache, memory)
        return self._prefill(x, q, k, v, qr, kr, int(start), cache, memory)

    def _prefill_setup(self, x, q, k, v, qr, kr, start, cache, memory, out=None, two_phase=False):
        """Operands of one layer prefill: bf16 inputs, sinks, the cache in device layout, output, workspace.
        ``out`` (optional): a contiguous fp32 [B,t,H,D] tensor the layer writes its output into."""
        B, t = x.shape[:2]
        H, G, D, W, S = self.H, self.G, self.D, self.window, self.sinks
        dev = x.device
        bf = torch.bfloat16
        xb, qb, kb, vb = (z.to(bf).contiguous() for z in (x, q, k, v))
        qrb, krb = qr.to(bf).contiguous(), kr.to(bf).contiguous()
        st = cache if cache is not None else {}
        # sinks: the first S positions, extended with this call's tokens below S (hibrit.py:369-373)
        sk, sv = st.get("sink_k"), st.get("sink_v")
        n_new = max(0, min(t, S - start))
        if n_new:
            nk, nv = krb[:, :, :n_new], vb[:, :n_new].transpose(1, 2)
            sk = nk if sk is None else torch.cat((sk.to(bf), nk), 2)
            sv = nv if sv is None else torch.cat((sv.to(bf), nv), 2)
        if sk is not None:
            sk, sv = sk.to(bf).contiguous(), sv.to(bf).contiguous()
        ns = 0 if sk is None else sk.shape[2]
        use_mem = bool(memory) and start + t > W
        rc = None
        if cache is not None:
            if "ring_k" not in cache:
                cache.update(ring_k=torch.zeros(B, G, W, D, device=dev, dtype=bf),
                             ring_v=torch.zeros(B, G, W, D, device=dev, dtype=bf),
                             ring_km=torch.zeros(B, W, G, D, device=dev, dtype=torch.float32),
                             ring_g=torch.zeros(B, W, G, device=dev, dtype=torch.float32),
                             ring_beta=torch.zeros(B, W, G, device=dev, dtype=torch.float32),
                             ring_pos=torch.full((W,), -1, device=dev, dtype=torch.int64))
            for key, dt in (("ring_k", bf), ("ring_v", bf), ("ring_km", torch.float32), ("ring_g", torch.float32),
                            ("ring_beta", torch.float32), ("ring_pos", torch.int64)):
                tns = cache[key]
                if tns.dtype != dt or not tns.is_contiguous() or tns.device != dev:
                    cache[key] = tns.to(device=dev, dtype=dt).contiguous()
            if use_mem:
                s0 = cache.get("S")
                if s0 is None:
                    cache["S"] = torch.zeros(B, G, D, D, device=dev, dtype=torch.float32)
                elif s0.dtype != torch.float32 or not s0.is_contiguous() or s0.device != dev:
                    cache["S"] = s0.to(device=dev, dtype=torch.float32).contiguous()
            Sst = cache["S"] if use_mem else _dummy_state(dev)
            rc = BfRingCache(ptr(cache["ring_k"]), ptr(cache["ring_v"]), ptr(cache["ring_km"]), ptr(cache["ring_g"]),
                             ptr(cache["ring_beta"]), ptr(cache["ring_pos"]), 0, 0, 0, 0, ptr(Sst))
        if out is not None:
            if tuple(out.shape) != (B, t, H, D) or out.dtype != torch.float32 or not out.is_contiguous():
                raise ValueError("out must be a contiguous fp32 tensor [B, t, H, D]")
            o = out
        else:
            o = torch.empty(B, t, H, D, device=dev, dtype=torch.float32)
        ring_case = cache is not None and start > 0
        nws = _lib.size("bf_layer_prefill_sp_workspace" if two_phase else "bf_layer_prefill_workspace", B, t, H, G, D,
                        W, 1 if ring_case else 0)
        ws = torch.empty(nws, dtype=torch.uint8, device=dev)
        return dict(args=(xb, qb, kb, vb, qrb, krb), B=B, t=t, start=start, rc=rc, sk=sk, sv=sv, ns=ns, o=o, ws=ws,
                    nws=nws, cache=cache)

    def _finish_cache(self, c):
        if c["cache"] is not None:
            c["cache"]["sink_k"], c["cache"]["sink_v"] = c["sk"], c["sv"]

    def _prefill(self, x, q, k, v, qr, kr, start, cache, memory, lse_out=None, out=None):
        c = self._prefill_setup(x, q, k, v, qr, kr, start, cache, memory, out)
        xb, qb, kb, vb, qrb, krb = c["args"]
        _lib.call("bf_bifrost_layer_prefill", ctypes_ref(self._struct), ptr(xb), ptr(qb), ptr(kb), ptr(vb), ptr(qrb),
                  ptr(krb), start, c["B"], c["t"], 0 if c["rc"] is None else ctypes_ref(c["rc"]), ptr(c["sk"]),
                  ptr(c["sv"]), c["ns"], 1 if memory else 0, ptr(c["o"]), ptr(lse_out), ptr(c["ws"]), c["nws"],
                  stream_handle())
        self._finish_cache(c)
        return c["o"]

    def student_varlen(self, x, q, k, v, qr, kr, cu_seqlens, memory: bool = True, caches=None, streams: int = 4):
        """The layer core over packed variable-length sequences: the T tokens of x [1,T,d],
        q [1,T,H,D], k/v [1,T,G,D], qr [1,H,T,D], kr [1,G,T,D] are n sequences, sequence i being tokens
        cu_seqlens[i] .. cu_seqlens[i+1] - 1.  Each sequence is its own prefill from an empty cache: its own
        positions from 0, sinks, window and ring, and a memory state that starts at zero (the reference runs
        ``_student`` once per sequence for this, heimdall/hibrit.py:363-424; it has no packed form).  Returns o
        [1,T,H,D] fp32.  ``caches`` (optional list of n dicts) receives each sequence's cache, ready for decode.

        ``cu_seqlens`` is read on the host (a list or tensor of n+1 cumulative lengths; a device tensor costs one
        copy to the host).  The per-sequence fused prefills are issued on ``streams`` rotating streams: each one
        forks its window and memory chain onto the device's two side streams, so one sequence's window runs
        while the previous sequence's memory reads finish, and the outputs are written straight into the
        packed result."""
        check_cuda(x, q, k, v, qr, kr)
        cu = [int(c) for c in (cu_seqlens.tolist() if isinstance(cu_seqlens, torch.Tensor) else cu_seqlens)]
        if x.shape[0] != 1 or len(cu) < 2 or cu[0] != 0 or cu[-1] != x.shape[1] or \
                any(b < a for a, b in zip(cu, cu[1:])):
            raise ValueError("cu_seqlens must be non-decreasing from 0 to T (with batch size 1)")
        if caches is not None and len(caches) != len(cu) - 1:
            raise ValueError("caches needs one dict per sequence")
        dev = x.device
        T = x.shape[1]
        out = torch.empty(1, T, self.H, self.D, device=dev, dtype=torch.float32)
        cur = torch.cuda.current_stream(dev)
        pool = _varlen_streams(dev, max(1, int(streams)))
        for s_ in pool:
            s_.wait_stream(cur)
        for i, (a, b) in enumerate(zip(cu, cu[1:])):
            if b == a:
                if caches is not None:
                    caches[i].clear()
                continue
            s_ = pool[i % len(pool)]
            with torch.cuda.stream(s_):
                args = (x[:, a:b], q[:, a:b], k[:, a:b], v[:, a:b], qr[:, :, a:b].contiguous(),
                        kr[:, :, a:b].contiguous())
                cache = caches[i] if caches is not None else None
                if cache is not None:
                    cache.clear()
                self._prefill(*args, 0, cache, memory, out=out[:, a:b])
        for s_ in pool:
            cur.wait_stream(s_)
        out.record_stream(cur)
        for s_ in pool:
            out.record_stream(s_)
        return out

    def prefill_sp_begin(self, x, q, k, v, qr, kr, start: int, cache: dict):
        """First phase of a sequence-parallel layer prefill of this rank's tokens (``heimdall_b200.sp``):
        the memory inputs, the per-chunk products and this segment's state map.  ``cache`` holds the ring
        (the W tokens before ``start``) and the sinks; its "S" is replaced by the incoming state before
        ``prefill_sp_finish``.  Returns (M, N, handle): S_out = M S_in + N for the segment's write stream.

        The window attention of the segment is still running when this returns (it is joined by
        ``prefill_sp_finish``) and uses buffers that the handle holds; a handle dropped without
        ``prefill_sp_finish`` waits for the device before those buffers are released."""
        check_cuda(x, q, k, v, qr, kr)
        c = _SpHandle(self._prefill_setup(x, q, k, v, qr, kr, int(start), cache, True, two_phase=True))
        B, G, D = c["B"], self.G, self.D
        M = torch.empty(B, G, D, D, device=x.device, dtype=torch.float32)
        N = torch.empty_like(M)
        self._prefill_sp_call(c, 0, M, N)
        c["maps"] = (M, N)
        done = [False]
        c["_joined"] = done
        weakref.finalize(c, _sp_abandoned, x.device, done)
        return M, N, c

    def prefill_sp_finish(self, handle):
        """Second phase: the rest of the prefill from the incoming state now in ``cache["S"]``; returns o and
        leaves ``cache["S"]`` = M S_in + N, the state after the segment."""
        c = handle
        cache = c["cache"]
        if c["rc"] is not None and "S" in cache:
            c["rc"].S = ptr(cache["S"])
        self._prefill_sp_call(c, 1, *c["maps"])
        c["_joined"][0] = True
        self._finish_cache(c)
        return c["o"]

    def _prefill_sp_call(self, c, phase, M, N):
        xb, qb, kb, vb, qrb, krb = c["args"]
        _lib.call("bf_bifrost_layer_prefill_sp", ctypes_ref(self._struct), ptr(xb), ptr(qb), ptr(kb), ptr(vb),
                  ptr(qrb), ptr(krb), c["start"], c["B"], c["t"], 0 if c["rc"] is None else ctypes_ref(c["rc"]),
                  ptr(c["sk"]), ptr(c["sv"]), c["ns"], phase, ptr(M), ptr(N), ptr(c["o"]), None, ptr(c["ws"]),
                  c["nws"], stream_handle())

    def student_host(self, x, q, k, v, qr, kr, start: int = 0, cache=None, memory: bool = True,
                     chunk: int = 4096, out=None):
        """``student`` for inputs in host memory: returns o [B,T,H,D] fp32 in pinned host memory.

        The sequence is processed in chunks of ``chunk`` tokens (a prefill with a carried cache, which
        gives the result of one pass over the whole sequence: the cache holds exactly what the next
        tokens read), on three streams so that the host->device copy of chunk i+1, the layer on chunk i
        and the device->host copy of chunk i-1 overlap.  Inputs should be pinned for the copies to run
        asynchronously.  Layouts as ``student``: x [B,T,d], q [B,T,H,D], k/v [B,T,G,D], qr [B,H,T,D],
        kr [B,G,T,D].  When ``cache`` is None a private cache carries the chunks and is dropped.
        Returns after the output is in host memory."""
        dev = self.device
        B, T = x.shape[:2]
        H, G, D = self.H, self.G, self.D
        if T == 0:
            return torch.empty(B, 0, H, D, dtype=torch.float32).pin_memory() if out is None else out
        chunk = max(1, min(int(chunk), T))
        if out is None:
            out = torch.empty(B, T, H, D, dtype=torch.float32).pin_memory()
        st = cache if cache is not None else {}
        cur = torch.cuda.current_stream(dev)
        # persistent streams and staging slots: the caching allocator reuses blocks per stream, so fresh
        # streams on every call would make every call allocate (and free) device memory again
        s_in, s_comp, s_out = _host_streams(dev)
        for s_ in (s_in, s_comp, s_out):
            s_.wait_stream(cur)
        bf = torch.bfloat16
        key = (B, chunk, x.shape[2])
        if self._host_slots is None or self._host_slots[0] != key:
            def alloc():
                return (torch.empty(B, chunk, x.shape[2], device=dev, dtype=bf),
                        torch.empty(B, chunk, H, D, device=dev, dtype=bf),
                        torch.empty(B, chunk, G, D, device=dev, dtype=bf),
                        torch.empty(B, chunk, G, D, device=dev, dtype=bf),
                        torch.empty(B, H, chunk, D, device=dev, dtype=bf),
                        torch.empty(B, G, chunk, D, device=dev, dtype=bf))
            torch.cuda.synchronize(dev)
            self._host_slots = (key, [alloc(), alloc()])
        slots = self._host_slots[1]
        freed = [None, None]          # event: the layer has finished reading a slot
        outs = []
        t0 = 0
        for i, n in enumerate(_chunk_plan(T, chunk)):
            t1 = t0 + n
            sl = i % 2
            bx, bq, bk, bv, bqr, bkr = slots[sl]
            with torch.cuda.stream(s_in):
                if freed[sl] is not None:
                    s_in.wait_event(freed[sl])
                bx[:, :n].copy_(x[:, t0:t1], non_blocking=True)
                bq[:, :n].copy_(q[:, t0:t1], non_blocking=True)
                bk[:, :n].copy_(k[:, t0:t1], non_blocking=True)
                bv[:, :n].copy_(v[:, t0:t1], non_blocking=True)
                for b in range(B):          # head-major inputs: one contiguous run per (b, head)
                    for h in range(H):
                        bqr[b, h, :n].copy_(qr[b, h, t0:t1], non_blocking=True)
                    for g in range(G):
                        bkr[b, g, :n].copy_(kr[b, g, t0:t1], non_blocking=True)
                landed = torch.cuda.Event()
                landed.record(s_in)
            with torch.cuda.stream(s_comp):
                s_comp.wait_event(landed)
                if n == chunk:
                    args = (bx, bq, bk, bv, bqr, bkr)
                else:
                    args = (bx[:, :n], bq[:, :n], bk[:, :n], bv[:, :n], bqr[:, :, :n].contiguous(),
                            bkr[:, :, :n].contiguous())
                o = self._prefill(*args, start + t0, st, memory)
                freed[sl] = torch.cuda.Event()
                freed[sl].record(s_comp)
                done = torch.cuda.Event()
                done.record(s_comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                o.record_stream(s_out)
                if B == 1:
                    out[:, t0:t1].copy_(o, non_blocking=True)
                else:
                    for b in range(B):
                        out[b, t0:t1].copy_(o[b], non_blocking=True)
            outs.append(o)
            t0 = t1
        for s_ in (s_in, s_comp, s_out):
            cur.wait_stream(s_)
        s_out.synchronize()
        s_comp.synchronize()          # the staging slots are free for the next call
        return out

    def _decode(self, x, q, k, v, qr, kr, start, cache, memory):
        B = x.shape[0]
        H, G, D, W, S = self.H, self.G, self.D, self.window, self.sinks
        dev = x.device
        bf = torch.bfloat16
        xb = x.reshape(B, -1).to(bf).contiguous()
        qb = q.reshape(B, H, D).to(bf).contiguous()
        kb = k.reshape(B, G, D).to(bf).contiguous()
        vb = v.reshape(B, G, D).to(bf).contiguous()
        qrb = qr.reshape(B, H, D).to(bf).contiguous()
        krb = kr.reshape(B, G, D).to(bf).contiguous()
        # sinks: the first S tokens are kept (hibrit.py:369-373)
        if start < S:
            nk, nv = krb[:, :, None], vb[:, :, None]
            sk, sv = cache.get("sink_k"), cache.get("sink_v")
            cache["sink_k"] = nk if sk is None else torch.cat((sk.to(bf), nk), 2)
            cache["sink_v"] = nv if sv is None else torch.cat((sv.to(bf), nv), 2)
        sk, sv = cache.get("sink_k"), cache.get("sink_v")
        if sk is not None:
            sk, sv = sk.to(bf).contiguous(), sv.to(bf).contiguous()
            cache["sink_k"], cache["sink_v"] = sk, sv
        ns = 0 if sk is None else sk.shape[2]
        use_mem = bool(memory) and start + 1 > W
        for key, dt in (("ring_k", bf), ("ring_v", bf), ("ring_km", torch.float32), ("ring_g", torch.float32),
                        ("ring_beta", torch.float32), ("ring_pos", torch.int64)):
            tns = cache[key]
            if tns.dtype != dt or not tns.is_contiguous() or tns.device != dev:
                cache[key] = tns.to(device=dev, dtype=dt).contiguous()
        if use_mem:
            s0 = cache.get("S")
            if s0 is None:
                cache["S"] = torch.zeros(B, G, D, D, device=dev, dtype=torch.float32)
            elif s0.dtype != torch.float32 or not s0.is_contiguous():
                cache["S"] = s0.float().contiguous()
        Sst = cache.get("S") if use_mem else None
        rc = BfRingCache(ptr(cache["ring_k"]), ptr(cache["ring_v"]), ptr(cache["ring_km"]), ptr(cache["ring_g"]),
                         ptr(cache["ring_beta"]), ptr(cache["ring_pos"]), 0, ptr(sk), ptr(sv), ns,
                         ptr(Sst) if Sst is not None else ptr(_dummy_state(dev)))
        pos = torch.full((B,), start, device=dev, dtype=torch.int64)
        o = torch.empty(B, H, D, device=dev, dtype=torch.float32)
        nws = _lib.size("bf_layer_decode_workspace", B, H, G, D, W)
        ws = torch.empty(nws, dtype=torch.uint8, device=dev)
        _lib.call("bf_bifrost_layer_decode", ctypes_ref(self._struct), ptr(xb), ptr(qb), ptr(kb), ptr(vb), ptr(qrb),
                  ptr(krb), ptr(pos), B, ctypes_ref(rc), 1 if use_mem else 0, ptr(o), 0, ptr(ws), nws,
                  stream_handle())
        return o.reshape(B, 1, H, D)

    def decode_step(self, x, q, k, v, qr, kr, pos, cache: dict, memory: bool = True, lse=None, ws=None):
        """One decode token per sequence where every sequence has its own position (serving: a batch of
        sequences at different lengths).  The reference's ``_student`` with t == 1 (hibrit.py:363-424) is the
        case of one shared position; this is that step run for each sequence at once.

        x [B,d], q/qr [B,H,D], k/kr/v [B,G,D] (bf16 or castable); pos [B] int64 on the device (the new
        tokens' positions, not changed here).  ``cache`` holds the reference's keys on the device in kernel
        layout: ring_k/ring_v [B,G,W,D] bf16, ring_km [B,W,G,D], ring_g/ring_beta [B,W,G], ring_pos [B,W]
        (one ring position row per sequence; [W] when all sequences share it), sink_k/sink_v [B,G,ns,D] bf16
        with every sequence past its sinks (ns == sinks), and S [B,G,D,D]; it is updated in place.  ``lse``
        [B,H] fp32 receives the window log-sum-exp when given; ``ws`` is an optional reusable workspace of
        at least ``bf_layer_decode_workspace`` bytes.  Returns o [B,H,D] fp32."""
        check_cuda(x, q, k, v, qr, kr, pos)
        B = x.shape[0]
        H, G, D, W = self.H, self.G, self.D, self.window
        dev = x.device
        bf = torch.bfloat16
        args = [z.reshape(B, -1).to(bf).contiguous() for z in (x, q, k, v, qr, kr)]
        for key, dt in (("ring_k", bf), ("ring_v", bf), ("ring_km", torch.float32), ("ring_g", torch.float32),
                        ("ring_beta", torch.float32), ("ring_pos", torch.int64), ("S", torch.float32)):
            tns = cache[key]
            if tns.dtype != dt or not tns.is_contiguous() or tns.device != dev:
                raise ValueError(f"decode_step: cache[{key!r}] must be a contiguous {dt} tensor on {dev}")
        rp = cache["ring_pos"]
        if rp.dim() == 2 and tuple(rp.shape) != (B, W) or rp.dim() == 1 and rp.numel() != W:
            raise ValueError("decode_step: ring_pos must be [W] or [B, W]")
        sk, sv = cache.get("sink_k"), cache.get("sink_v")
        ns = 0 if sk is None else sk.shape[2]
        if sk is not None and (sk.dtype != bf or sv.dtype != bf or not sk.is_contiguous() or not sv.is_contiguous()):
            raise ValueError("decode_step: sinks must be contiguous bf16 [B,G,ns,D]")
        p = pos.to(device=dev, dtype=torch.int64).contiguous()
        rc = BfRingCache(ptr(cache["ring_k"]), ptr(cache["ring_v"]), ptr(cache["ring_km"]), ptr(cache["ring_g"]),
                         ptr(cache["ring_beta"]), ptr(rp), W if rp.dim() == 2 else 0, ptr(sk), ptr(sv), ns,
                         ptr(cache["S"]))
        o = torch.empty(B, H, D, device=dev, dtype=torch.float32)
        nws = _lib.size("bf_layer_decode_workspace", B, H, G, D, W)
        if ws is None or ws.numel() < nws:
            ws = torch.empty(nws, dtype=torch.uint8, device=dev)
        _lib.call("bf_bifrost_layer_decode", ctypes_ref(self._struct), *(ptr(z) for z in args), ptr(p), B,
                  ctypes_ref(rc), 1 if memory else 0, ptr(o), ptr(lse), ptr(ws), ws.numel(), stream_handle())
        return o


_DUMMY = {}
_STREAMS = {}


def _chunk_plan(T: int, chunk: int) -> list:
    """Chunk lengths for the host-buffer prefill: equal chunks, the last one ragged (a ramp of smaller chunks
    at both ends measured slower on B200: the per-chunk fixed costs outweigh the shorter fill and drain)."""
    return [min(chunk, T - t0) for t0 in range(0, T, chunk)]


_VARLEN_STREAMS = {}


def _varlen_streams(dev, n: int):
    """n caller streams per device for the packed-sequence prefill (kept for the process)."""
    key = (str(dev), n)
    if key not in _VARLEN_STREAMS:
        _VARLEN_STREAMS[key] = tuple(torch.cuda.Stream(dev) for _ in range(n))
    return _VARLEN_STREAMS[key]


def _host_streams(dev):
    """Three streams per device for the host-buffer prefill: copies in, the layer, copies out."""
    key = str(dev)
    if key not in _STREAMS:
        _STREAMS[key] = tuple(torch.cuda.Stream(dev) for _ in range(3))
    return _STREAMS[key]


def _dummy_state(dev):
    # a 16-byte-aligned placeholder for the state pointer when memory is off (never read or written)
    key = str(dev)
    if key not in _DUMMY:
        _DUMMY[key] = torch.zeros(4, device=dev, dtype=torch.float32)
    return _DUMMY[key]


def ctypes_ref(s):
    """Address of a ctypes struct, for the c_void_p struct-pointer arguments (the struct outlives the call)."""
    import ctypes
    return ctypes.addressof(s)


class _SpHandle(dict):
    """The state of a sequence-parallel prefill between its two phases (a dict that can carry a finalizer)."""


def _sp_abandoned(device, done):
    # a first phase whose second never ran: its window kernel may still use the handle's buffers
    if not done[0]:
        torch.cuda.synchronize(device)

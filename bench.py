#!/usr/bin/env python
"""Bifrost-layer benchmark on B200 (the headline is config 3 at 128K).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (``value``): one converted Bifrost layer prefill of ONE 131072-token sequence (B=1, 24 query / 4 KV
heads, head dim 256, window 2048 + 4 sinks, hidden size 5120, bf16 inputs, fp32 state and outputs, from an empty
cache), split evenly over the N GPUs (sequence parallelism: halo exchange, per-segment state maps all-gathered
and prefix-folded over NCCL, then each rank's prefill; ``heimdall_b200.sp.student_sp``).  N = 1 is one ordinary
prefill (``BifrostLayer.student`` -> ``bf_bifrost_layer_prefill``).  The total work is fixed, so the scaling is
strong and the driver's per-N values give the sequence-parallel efficiency.  Inputs are synthetic (seeded,
RMS-normalised q/k/v) and larger than L2 (5.4 GB per step on one GPU), so no L2 flush is needed.  Timed with
CUDA events over exactly --steps steps after --warmup, max over ranks; rank 0 prints one JSON line.

Extra keys: ``config1`` (T = 32768 on each GPU: stage times, the layer roofline) and
``roofline`` (its dominant kernel, the window attention, timed live on its stream; peak = the measured burst
bf16 figure when the timed clocks sat at max, else the sustained one), ``layer_roofline`` (all algorithmic
FLOPs of the headline step), ``cpu_baseline`` (the CPU oracle port in the reference's own form on a bounded
sample), ``e2e`` (the headline through the public API from pinned host buffers, copies inside the timed
region), ``sp_131k`` (N > 1: a per-rank timeline of one step and an in-bench parity check against one prefill
of the whole sequence on one GPU), ``sp_1m`` (config 3 at T = 1048576, same), ``decode`` (64
sequences x 12 layers, sharded over the N GPUs), ``delta_rule`` (configs 0 and 4: the chunked delta-rule op),
``interchange`` (N = 1: the llama.cpp state rows of config 2's decode cache, packed and unpacked),
``retrieval`` (N = 1: a kept full-attention layer's retrieval decode at 128K context), ``clocks``
(nvidia-smi samples during the timed region) and ``gpu_launches``.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

H, G, D, DM, W, S = 24, 4, 256, 5120, 2048, 4
R = H // G
METRIC = "Bifrost-layer prefill tok/s @32K/128K, decode us/token; % of roofline"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# ---------------------------------------------------------------------------------------------- helpers
def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def rms(z):
    return z * torch.rsqrt(z.float().square().mean(-1, keepdim=True) + 1e-6).to(z.dtype)


def make_inputs(T, seed, device, B=1):
    gen = torch.Generator(device=device).manual_seed(seed)
    bf = torch.bfloat16
    r = lambda *s: torch.randn(*s, generator=gen, device=device, dtype=torch.float32)
    x = r(B, T, DM).to(bf)
    q = rms(r(B, T, H, D)).to(bf)
    k = rms(r(B, T, G, D)).to(bf)
    v = rms(r(B, T, G, D)).to(bf)
    qr = rms(r(B, H, T, D)).to(bf)
    kr = rms(r(B, G, T, D)).to(bf)
    return x, q, k, v, qr, kr


def window_standalone_ms(inputs, reps=5):
    """The window op alone (``bf_window_attn_fwd``: V^T staging + the kernel, persistent launch) on the step's
    resident inputs, CUDA events on the current stream: the kernel's own speed, beside its stage time inside the
    layer step (where it shares the SMs with the memory chain)."""
    from heimdall_b200 import functional as F_
    x, q, k, v, qr, kr = inputs
    sk, sv = kr[:, :, :S].contiguous(), v[:, :S].transpose(1, 2).contiguous()
    vext = v.transpose(1, 2)
    run = lambda: F_.window_attention(qr, kr, vext, 0, 0, S, W, sk, sv)
    run()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        run()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def make_layer(device, seed=0):
    """Config 1 parameters: convert(2048, 4, archival=1, "long") with seed 0, then mix / mix_lse / mem_scale
    ~ N(0, 0.02)."""
    from heimdall_b200 import BifrostLayer
    gen = torch.Generator().manual_seed(seed)
    L = BifrostLayer.converted(H, G, D, DM, W, S, archival=1, mem_init="long", generator=gen, device=device)
    n = lambda *s: torch.randn(*s, generator=gen) * 0.02
    L.p["mix_w"].copy_(n(H, DM))
    L.p["mix_b"].copy_(n(H))
    L.p["mix_lse"].copy_(n(H))
    L.p["mem_scale"].copy_(n(H))
    L.refresh()
    return L


def layer_flops(T):
    """Algorithmic FLOPs of one layer prefill from an empty cache (counting rules of the survey, section 8d):
    window 4 H D per (query, valid key) pair, delta rule G (6CD + 4D^2 + R(4CD + 2D^2)) per write step (C = 64),
    projections 2D^2(H+G) + 2d(2G+H) per token."""
    # valid keys of the query at position t: min(S, t+1) sinks plus the window keys max(S, t-W+1) .. t
    def win_keys(t0, t1):    # sum over t in [t0, t1) of the window keys, for t >= S (lo = max(S, t-W+1))
        total = 0
        a = max(t0, S)
        b1 = min(t1, S + W - 1)              # t - W + 1 <= S: lo = S, keys = t - S + 1
        if b1 > a:
            total += (b1 - a) * (a + b1 - 1) // 2 - (S - 1) * (b1 - a)
        a2 = max(t0, S + W - 1, a)           # lo = t - W + 1: keys = W
        if t1 > a2:
            total += (t1 - a2) * W
        return total
    sinks = sum(min(S, t + 1) for t in range(min(T, S))) + S * max(0, T - S)
    win = win_keys(0, T) + sinks
    win_flops = 4 * H * D * win
    C = 64
    delta_per_tok = G * (6 * C * D + 4 * D * D + R * (4 * C * D + 2 * D * D))
    delta_flops = delta_per_tok * max(0, T - W)
    proj_flops = (2 * D * D * (H + G) + 2 * DM * (2 * G + H)) * T
    return win_flops, delta_flops, proj_flops


class ClockSampler:
    """nvidia-smi samples (200 ms) while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = Path(f"/tmp/bf_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.idx)], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), smax=float(parts[2]), power=float(parts[3]),
                                 hw=parts[5], hwt=parts[6], swt=parts[7], swp=parts[8]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        pmax = max(r["power"] for r in rows)
        load = [r for r in rows if r["power"] >= 0.5 * pmax] or rows
        reasons = set()
        for r in load:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"), ("swt", "sw_thermal_slowdown"),
                              ("swp", "sw_power_cap")):
                if r[key].lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in load), "sm_max_mhz": max(r["smax"] for r in load),
                "power_w_max": pmax, "samples": len(load), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------------------------- our arm
def run_prefill(L, inputs, steps, warmup, T, dist_ctx, stage_names):
    from heimdall_b200 import _lib
    x, q, k, v, qr, kr = inputs
    for _ in range(warmup):
        L.student(x, q, k, v, qr, kr, 0, None)
    torch.cuda.synchronize()
    nst = len(stage_names)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2 * nst)] for _ in range(steps)]
    for es in evs:                       # torch creates the CUDA event on its first record
        for e in es:
            e.record()
    torch.cuda.synchronize()
    handles = [ctypes_array([e.cuda_event for e in es]) for es in evs]
    barrier(dist_ctx)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for i in range(steps):
        _lib.call("bf_stage_events", handles[i], nst)
        L.student(x, q, k, v, qr, kr, 0, None)
    end.record()
    torch.cuda.synchronize()
    _lib.call("bf_stage_events", None, 0)
    ms = start.elapsed_time(end)
    stage_ms = {}
    for j, name in enumerate(stage_names):
        vals = []
        for es in evs:
            try:
                vals.append(es[2 * j].elapsed_time(es[2 * j + 1]))
            except RuntimeError:
                pass
        if vals:
            stage_ms[name] = sum(vals) / len(vals)
    return ms, stage_ms


def ctypes_array(handles):
    import ctypes
    arr = (ctypes.c_void_p * len(handles))(*handles)
    return arr


SP_STAGES = ["x_proj", "head_proj", "gdn_p1", "gdn_p2", "gdn_p3", "window_prep", "window", "cache"]


def _sp_stage_hook(handles):
    """phase_hook for student_sp: per-phase stage events (phase 0: memory inputs, P1, the state-map scan, the
    window; phase 1: the scan from the incoming state, the memory reads)."""
    from heimdall_b200 import _lib

    def hook(phase):
        _lib.call("bf_stage_events", handles[phase], len(SP_STAGES))
    return hook


def run_sp(L, device, ctx, T_total, steps=5, warmup=2):
    """one sequence of T_total tokens split over the ranks (heimdall_b200.sp.student_sp:
    halo exchange, segment state maps, all-gather, prefix fold, then each rank's prefill).  At N=1 the
    same sequence is one ordinary prefill.  Max over ranks of the device time.

    At N > 1 it also reports each rank's timeline of one instrumented step (ms from the step's start: the
    student_sp marks and the kernels' stage events of both phases) and checks parity in the bench: rank 0
    runs the whole sequence as one prefill on its own GPU and compares the last rank's final state
    (rel-L2 <= 1e-3) and its last 2048 outputs (rel-L2 <= 2e-3), both sent to rank 0."""
    from heimdall_b200 import _lib, sp
    world, rank = ctx["world"], ctx["rank"]
    T = T_total // world
    ins = make_inputs(T, seed=11 + rank, device=device)
    gr = None
    if world > 1:   # timed: the captured step (StudentSPGraph); the instrumented step below runs eagerly
        gr = sp.StudentSPGraph(L, *ins, warmup=warmup)
        timed = gr.replay
        step = lambda **kw: sp.student_sp(L, *ins, **kw)
    else:
        timed = lambda: L.student(*ins, 0, {})
        for _ in range(warmup):
            timed()
    torch.cuda.synchronize()
    barrier(ctx)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        timed()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / steps], device=device)
    if world > 1:
        gr.check()
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    res = {"workload": f"BASELINE config 3: one sequence of {T_total} tokens split over {world} GPU(s) "
                       f"({T} per GPU), from an empty cache", "T_total": T_total, "ms_per_step": ms,
           "value": T_total / (ms / 1e3), "unit": "tok/s", "steps": steps, "warmup": warmup}
    if world == 1:
        del ins
        return res
    # one instrumented step: per-rank timeline
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2 * len(SP_STAGES))] for _ in range(2)]
    for es in evs:
        for e in es:
            e.record()
    torch.cuda.synchronize()
    handles = [ctypes_array([e.cuda_event for e in es]) for es in evs]
    timeline = []
    barrier(ctx)
    step(timeline=timeline, phase_hook=_sp_stage_hook(handles))
    torch.cuda.synchronize()
    _lib.call("bf_stage_events", None, 0)
    o, cache = gr.o, gr.cache          # parity below is checked on the timed (graph) step's results
    t0 = timeline[0][1]
    marks = {lab: round(t0.elapsed_time(ev), 4) for lab, ev in timeline}
    stages = {}
    for ph, es in enumerate(evs):
        for j, name in enumerate(SP_STAGES):
            try:
                stages[f"p{ph}.{name}"] = [round(t0.elapsed_time(es[2 * j]), 4), round(t0.elapsed_time(es[2 * j + 1]), 4)]
            except RuntimeError:
                pass
    per_rank = [None] * world
    torch.distributed.all_gather_object(per_rank, {"rank": rank, "marks_ms": marks, "stages_ms": stages})
    res["timeline"] = per_rank
    res["timeline_note"] = ("ms from the start of one instrumented step (eager, not the captured graph that is "
                            "timed) on each rank; marks are student_sp's steps "
                            "on its stream, stages are [begin, end] of the kernels of phase 0 (memory inputs, P1, "
                            "state-map scan, window) and phase 1 (scan from the incoming state, memory reads)")
    # parity: the last rank's final state and last outputs against one pass over the whole sequence on rank 0
    last = world - 1
    n_cmp = 2048
    if rank == last:
        torch.distributed.send(cache["S"].contiguous(), 0)
        torch.distributed.send(o[:, -n_cmp:].contiguous(), 0)
    elif rank == 0:
        S_last = torch.empty_like(cache["S"])
        o_last = torch.empty(o.shape[0], n_cmp, *o.shape[2:], device=device, dtype=o.dtype)
        torch.distributed.recv(S_last, last)
        torch.distributed.recv(o_last, last)
    del o, cache, ins
    gr = None                          # the graph holds NCCL calls: released before any process-group teardown
    torch.cuda.synchronize()
    if rank == 0:
        torch.cuda.empty_cache()
        full = [torch.empty(1, T_total, *shape[2:], device=device, dtype=torch.bfloat16) if i < 4 else
                torch.empty(1, shape[1], T_total, shape[3], device=device, dtype=torch.bfloat16)
                for i, shape in enumerate(_input_shapes(T))]
        for r in range(world):
            part = make_inputs(T, seed=11 + r, device=device)
            for i, z in enumerate(part):
                if i < 4:
                    full[i][:, r * T:(r + 1) * T] = z
                else:
                    full[i][:, :, r * T:(r + 1) * T] = z
            del part
        cache1 = {}
        o1 = L.student(*full, 0, cache1)
        torch.cuda.synchronize()
        rel = lambda a_, b_: float((a_.double() - b_.double()).norm() / b_.double().norm())
        es = rel(S_last, cache1["S"])
        eo = rel(o_last, o1[:, -n_cmp:])
        res["parity"] = {"against": "one prefill of the whole sequence on one GPU", "state_rel_l2": es,
                         "state_tol": 1e-3, "last_outputs_rel_l2": eo, "outputs_tol": 2e-3,
                         "outputs_compared": f"the last {n_cmp} tokens of rank {last}", "ok": es <= 1e-3 and eo <= 2e-3}
        del full, o1, cache1
        torch.cuda.empty_cache()
    barrier(ctx)
    return res


def _input_shapes(T, B=1):
    return [(B, T, DM), (B, T, H, D), (B, T, G, D), (B, T, G, D), (B, H, T, D), (B, G, T, D)]


def _time_device(fn, steps, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def run_delta_configs(device, steps=10, warmup=3):
    """BASELINE configs 0 and 4 (the chunked delta-rule op alone, ``delta_rule`` / ``delta_rule_gqa``):
    config 0 = B=1, 4 heads, T=4096, D=256, fp32 inputs (q, k unit-norm, v ~ N(0,1), beta = sigmoid(N(0,1)),
    g = -e^{A_log} softplus(a) with A_log ~ U(-4,0), a ~ N(0,1)); config 4 = 8 packed sequences of
    round(exp U[ln 2048, ln 65536]) tokens (seed 0) with cu_seqlens, 4 KV heads x 6 query heads, fixed-rate
    decays (half-lives logspace(log10 2048, 6, 4), the last head archival)."""
    import torch.nn.functional as F
    from heimdall_b200.functional import delta_rule, delta_rule_gqa
    out = {}
    torch.manual_seed(0)
    Hc, Tc = 4, 4096
    q = F.normalize(torch.randn(1, Tc, Hc, D), dim=-1)
    k = F.normalize(torch.randn(1, Tc, Hc, D), dim=-1)
    v = torch.randn(1, Tc, Hc, D)
    beta = torch.sigmoid(torch.randn(1, Tc, Hc))
    A_log = torch.empty(Hc).uniform_(-4, 0)
    g = -A_log.exp() * F.softplus(torch.randn(1, Tc, Hc))
    args = [z.to(device) for z in (q, k, v, g, beta)]
    ms = _time_device(lambda: delta_rule(*args, 64, None), steps, warmup)
    out["config0"] = {"workload": "BASELINE config 0: delta rule, B=1, H=4, T=4096, D=256, fp32 inputs",
                      "value": Tc / (ms / 1e3), "unit": "tok/s", "ms_per_step": ms}
    gen = torch.Generator().manual_seed(0)
    lens = torch.exp(torch.empty(8).uniform_(math.log(2048), math.log(65536), generator=gen)).round().long()
    T4 = int(lens.sum())
    cu = torch.cat((torch.zeros(1, dtype=torch.long), lens.cumsum(0))).to(torch.int32)
    Gc, Rc = 4, 6
    life = torch.logspace(math.log10(2048), 6.0, Gc)
    gfix = -(math.log(2.0) / life)
    gfix[-1] = 0.0
    q4 = F.normalize(torch.randn(1, T4, Gc, Rc, D, generator=gen), dim=-1) * D ** -0.5
    k4 = F.normalize(torch.randn(1, T4, Gc, D, generator=gen), dim=-1)
    v4 = torch.randn(1, T4, Gc, D, generator=gen).to(torch.bfloat16)
    b4 = torch.sigmoid(torch.randn(1, T4, Gc, generator=gen))
    g4 = gfix.expand(1, T4, Gc).contiguous()
    args4 = [z.to(device) for z in (q4, k4, v4, g4, b4)]
    cud = cu.to(device)
    ms4 = _time_device(lambda: delta_rule_gqa(*args4, 64, None, cu_seqlens=cud), steps, warmup)
    out["config4"] = {"workload": f"BASELINE config 4, the delta-rule op alone: 8 packed sequences ({lens.tolist()} "
                                  f"tokens, {T4} total) with cu_seqlens, 4 KV x 6 query heads, D=256",
                      "value": T4 / (ms4 / 1e3), "unit": "tok/s", "ms_per_step": ms4}
    del args4
    out["config4_layer"] = run_config4_layer(device, lens.tolist(), steps=max(3, steps // 2), warmup=2)
    return out


def run_config4_layer(device, lens, steps=5, warmup=2):
    """BASELINE config 4 as the full layer (window + memory + gate): the 8 packed sequences through
    ``BifrostLayer.student_varlen``, each with its own positions, sinks, ring and a state reset at its start;
    fixed-rate decays (the x-dependent decay input zeroed) with half-lives logspace(log10 2048, 6, 4) and the
    last KV head archival; inputs as config 1."""
    L = make_layer(device, seed=4)
    life = torch.logspace(math.log10(2048), 6.0, G, device=device)
    L.p["ab_w"][:G].zero_()
    L.p["ab_b"][:G].zero_()
    L.p["A_log"].copy_((math.log(2.0) / life / torch.nn.functional.softplus(L.p["dt_bias"])).log())
    L.p["decay_mask"].fill_(1.0)
    L.p["decay_mask"][-1] = 0.0
    L.refresh()
    T = sum(lens)
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    ins = make_inputs(T, seed=41, device=device)
    ms = _time_device(lambda: L.student_varlen(*ins, cu), steps, warmup)
    win_f = sum(sum(layer_flops_split(n)) for n in lens)
    del ins
    return {"workload": f"BASELINE config 4, the full layer: 8 packed sequences ({lens} tokens, {T} total), "
                        f"window + memory + gate, per-sequence state reset", "value": T / (ms / 1e3), "unit": "tok/s",
            "ms_per_step": ms, "achieved_tflops": win_f / (ms * 1e-3) / 1e12}


def layer_flops_split(T):
    return layer_flops(T)


def run_decode(device, ctx, steps=256, warmup=8, nseq=64, nlayers=12):
    """64 sequences at positions U[4K, 128K], 12 stacked layers, one token per sequence per
    step; the whole 12-layer step is captured in a CUDA graph and replayed.  With N ranks the sequences are
    sharded (64 / N per GPU, no collective: sequences are independent); the step time is the max over ranks and
    the per-token figures are for the whole batch."""
    world, rank = ctx["world"], ctx["rank"]
    nseq_total = nseq
    nseq = max(1, nseq // world)
    from heimdall_b200 import _lib
    from heimdall_b200.layer import ctypes_ref
    from heimdall_b200.structs import BfRingCache
    from heimdall_b200.functional import ptr
    gen = torch.Generator(device=device).manual_seed(2 + 1000 * rank)
    bf = torch.bfloat16
    r = lambda *s: torch.randn(*s, generator=gen, device=device)
    layers, caches, ins, outs, wss = [], [], [], [], []
    pos = torch.randint(4096, 131072, (nseq,), generator=gen, device=device, dtype=torch.int64)
    for li in range(nlayers):
        L = make_layer(device, seed=100 + li)
        layers.append(L)
        ring_pos = (pos[:, None] - W + torch.arange(W, device=device)[None]).to(torch.int64)
        # slot of position p is p % W: scatter the W most recent positions into their slots
        rp = torch.empty(nseq, W, dtype=torch.int64, device=device)
        rp.scatter_(1, ring_pos % W, ring_pos)
        c = dict(ring_k=rms(r(nseq, G, W, D)).to(bf), ring_v=rms(r(nseq, G, W, D)).to(bf),
                 ring_km=torch.nn.functional.normalize(r(nseq, W, G, D), dim=-1),
                 ring_g=-torch.rand(nseq, W, G, generator=gen, device=device) * 0.01,
                 ring_beta=torch.rand(nseq, W, G, generator=gen, device=device), ring_pos=rp,
                 sink_k=rms(r(nseq, G, S, D)).to(bf), sink_v=rms(r(nseq, G, S, D)).to(bf),
                 S=r(nseq, G, D, D) * 0.02)
        caches.append(c)
        ins.append(dict(x=r(nseq, DM).to(bf), q=rms(r(nseq, H, D)).to(bf), k=rms(r(nseq, G, D)).to(bf),
                        v=rms(r(nseq, G, D)).to(bf), qr=rms(r(nseq, H, D)).to(bf), kr=rms(r(nseq, G, D)).to(bf)))
        outs.append(torch.empty(nseq, H, D, device=device))
        n = _lib.size("bf_layer_decode_workspace", nseq, H, G, D, W)
        wss.append(torch.empty(n, dtype=torch.uint8, device=device))
    structs = [BfRingCache(ptr(c["ring_k"]), ptr(c["ring_v"]), ptr(c["ring_km"]), ptr(c["ring_g"]),
                           ptr(c["ring_beta"]), ptr(c["ring_pos"]), W, ptr(c["sink_k"]), ptr(c["sink_v"]), S,
                           ptr(c["S"])) for c in caches]
    stream = torch.cuda.Stream(device=device)

    def step():
        sh = torch.cuda.current_stream().cuda_stream
        for L, c, i, o, ws in zip(layers, structs, ins, outs, wss):
            _lib.call("bf_bifrost_layer_decode", ctypes_ref(L.struct), ptr(i["x"]), ptr(i["q"]), ptr(i["k"]),
                      ptr(i["v"]), ptr(i["qr"]), ptr(i["kr"]), ptr(pos), nseq, ctypes_ref(c), 1, ptr(o), 0, ptr(ws),
                      ws.numel(), sh)
        pos.add_(1)

    with torch.cuda.stream(stream):
        for _ in range(warmup):
            step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    torch.cuda.synchronize()
    # per-kernel stage times of one layer (eager, same stream)
    NST = 12
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * NST)]
    for e in ev:
        e.record()
    torch.cuda.synchronize()
    barrier(ctx)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        a.record()
        for _ in range(steps):
            graph.replay()
        b.record()
    torch.cuda.synchronize()
    t_ = torch.tensor([a.elapsed_time(b) * 1e3 / steps], device=device)
    if world > 1:
        torch.distributed.all_reduce(t_, op=torch.distributed.ReduceOp.MAX)
    us_step = float(t_.item())
    # live per-kernel timing of the state update and the window (eager step with stage events)
    handles = ctypes_array([e.cuda_event for e in ev])
    names = {0: "x_proj", 1: "head_proj", 10: "gather", 8: "state_update", 9: "window_split", 11: "combine"}
    samples = {n: [] for n in names.values()}
    layer_us = []
    with torch.cuda.stream(stream):
        for _ in range(4):
            for L, c, i, o, ws in zip(layers, structs, ins, outs, wss):
                _lib.call("bf_stage_events", handles, NST)
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record()
                _lib.call("bf_bifrost_layer_decode", ctypes_ref(L.struct), ptr(i["x"]), ptr(i["q"]), ptr(i["k"]),
                          ptr(i["v"]), ptr(i["qr"]), ptr(i["kr"]), ptr(pos), nseq, ctypes_ref(c), 1, ptr(o), 0,
                          ptr(ws), ws.numel(), stream.cuda_stream)
                e1.record()
                torch.cuda.synchronize()
                layer_us.append(e0.elapsed_time(e1) * 1e3)
                for j, n in names.items():
                    samples[n].append(ev[2 * j].elapsed_time(ev[2 * j + 1]) * 1e3)
    _lib.call("bf_stage_events", None, 0)
    st_us, win_us = samples["state_update"], samples["window_split"]
    del graph
    state_bytes = 2 * nseq * G * D * D * 4
    win_bytes = nseq * G * (W + S) * D * 2 * 2
    pk, _ = peaks()
    su = statistics.fmean(st_us)   # event ticks are about 1 us: the mean of the samples resolves below that
    wu = statistics.fmean(win_us)
    per_layer_bytes = state_bytes + win_bytes
    return {"config": f"{nseq_total} sequences x {nlayers} layers ({nseq} per GPU on {world} GPU(s)), positions "
                      f"U[4096,131072), {steps} graph-replayed steps",
            "us_per_step": us_step, "us_per_token": us_step / nseq_total, "tokens_per_s": nseq_total / (us_step * 1e-6),
            "per_gpu_note": "state_update / window / step_roofline are for one GPU's shard (rank 0)",
            "state_update": {"us": su, "bytes": state_bytes, "achieved_gbs": state_bytes / (su * 1e-6) / 1e9,
                             "peak_gbs": pk["hbm_gbs"], "frac": state_bytes / (su * 1e-6) / 1e9 / pk["hbm_gbs"]},
            "window": {"us": wu, "bytes": win_bytes, "achieved_gbs": win_bytes / (wu * 1e-6) / 1e9,
                       "frac": win_bytes / (wu * 1e-6) / 1e9 / pk["hbm_gbs"], "kernel": "window split (combine apart)"},
            "stage_us": {n: statistics.fmean(v) for n, v in samples.items()},
            "eager_layer_us": statistics.fmean(layer_us),
            "step_roofline": {"bytes": per_layer_bytes * nlayers,
                              "frac": per_layer_bytes * nlayers / (us_step * 1e-6) / 1e9 / pk["hbm_gbs"]}}


def run_retrieval(device, nseq=16, n=131072, steps=20, warmup=3):
    """Retrieval decode of a kept full-attention layer (HybridAttention._teacher with set_retrieval defaults:
    k = 16 blocks of 64, window 2048, 4 sinks) for nseq sequences at context n: block bounds from the summaries,
    top-16 selection, exact attention over sinks + selected blocks + window.  HBM-bound: algorithmic bytes = the
    summaries of the candidate blocks plus every attended key and value, read once."""
    from heimdall_b200 import _lib
    from heimdall_b200.functional import ptr
    Sk, Wk, Lk, Kk = 4, 2048, 64, 16
    gen = torch.Generator(device=device).manual_seed(11)
    bf = torch.bfloat16
    k = torch.randn(nseq, G, n, D, generator=gen, device=device, dtype=bf)
    v = torch.randn(nseq, G, n, D, generator=gen, device=device, dtype=bf)
    nbcap = (n - Sk) // Lk
    kmin = torch.empty(nseq, G, nbcap, D, device=device, dtype=bf)
    kmax = torch.empty_like(kmin)
    _lib.call("bf_ret_summarize", ptr(k), n, nseq, G, D, Sk, Lk, 0, nbcap, ptr(kmin), ptr(kmax), nbcap, None)
    q = torch.randn(nseq, H, D, generator=gen, device=device, dtype=bf)
    o = torch.empty(nseq, H, D, device=device)
    nws = _lib.size("bf_ret_decode_workspace", nseq, H, G, D, n, Sk, Wk, Lk, Kk)
    ws = torch.empty(nws, dtype=torch.uint8, device=device)
    call = lambda: _lib.call("bf_ret_decode", ptr(q), ptr(k), ptr(v), n, ptr(kmin), ptr(kmax), nbcap, nseq, H, G, D,
                             n, Sk, Wk, Lk, Kk, ptr(o), ptr(ws), nws,
                             torch.cuda.current_stream(device).cuda_stream)
    ms = _time_device(call, steps, warmup)
    nc = (n - Wk - Sk) // Lk
    nk = Sk + Kk * Lk + (n - Sk - nc * Lk)
    nbytes = nseq * G * (2 * nc * D * 2 + 2 * nk * D * 2) + nseq * H * D * (2 + 4)
    pk, _ = peaks()
    del k, v
    return {"workload": f"{nseq} sequences at context {n}, one kept layer (24 query / 4 KV heads, D=256): "
                        f"retrieval decode, top-{Kk} blocks of {Lk} + window {Wk} + {Sk} sinks ({nk} keys attended)",
            "us_per_step": ms * 1e3, "us_per_token": ms * 1e3 / nseq, "bytes": nbytes,
            "achieved_gbs": nbytes / (ms * 1e-3) / 1e9, "frac": nbytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"]}


def run_backward(device, T=8192, steps=3, warmup=3):
    """Backward of ``delta_rule_gqa`` as seq_loss (motor.py:149-193) takes it: one segment of the conversion
    engine's length (8192 tokens), 4 KV heads x 6 query heads, D = 256, fp32, with an initial state and the
    final state's gradient.  The recurrence is sequential in the tokens (fp32, 32 CTAs of 8 value columns per
    KV head); the figure that bounds it is the dependent chain per token, so the leg reports microseconds per
    token beside the forward's time on the same inputs and the bytes the kernel moves (checkpoints, the
    per-chunk state scratch, the per-token partials)."""
    from heimdall_b200.functional import delta_rule_gqa, delta_rule_gqa_backward
    gen = torch.Generator(device=device).manual_seed(5)
    r = lambda *s: torch.randn(*s, generator=gen, device=device)
    q = torch.nn.functional.normalize(r(1, T, G, R, D), dim=-1) * D ** -0.5
    k = torch.nn.functional.normalize(r(1, T, G, D), dim=-1)
    v = r(1, T, G, D)
    g = -torch.rand(1, T, G, generator=gen, device=device) * 0.1
    beta = torch.rand(1, T, G, generator=gen, device=device)
    s0 = r(1, G, D, D) * 0.05
    do = r(1, T, G, R, D)
    dsT = r(1, G, D, D) * 0.05
    bwd_ms = _time_device(lambda: delta_rule_gqa_backward(q, k, v, g, beta, s0, do, dsT), steps, warmup)
    with torch.no_grad():
        fwd_ms = _time_device(lambda: delta_rule_gqa(q, k, v, g, beta, 64, s0), steps, warmup)
    state = G * D * D * 4
    ncta, E = D // 8, (R + 1) * D + 2          # CTAs of 8 value columns per KV head
    nbytes = (T // 64) * state * 2 + T * state * 2 + T * G * ncta * E * 4 * 2 + T * G * (R * D * 2 + 3 * D) * 4 * 3
    return {"workload": f"one {T}-token segment, {G} KV heads x {R} query heads, D={D}, fp32: dq, dk, dv, dg, dbeta, "
                        "ds0 from dL/do and dL/dS_T",
            "bwd_ms": bwd_ms, "fwd_ms": fwd_ms, "us_per_token": bwd_ms * 1e3 / T, "bytes": nbytes,
            "achieved_gbs": nbytes / (bwd_ms * 1e-3) / 1e9, "bound": "latency (sequential in tokens)"}


def run_interchange(device, nseq=64, steps=20, warmup=3):
    """The llama.cpp state-row interchange at config-2 geometry (64 sequences, W = 2048, one layer): pack the
    decode cache into the port's rows and unpack them again.  Both are HBM-bound copies (rows 43.7 MB per
    sequence); algorithmic bytes = every byte read plus every byte written once."""
    from heimdall_b200.interchange import llama_state_floats, pack_llama_state, unpack_llama_state
    L = make_layer(device, seed=7)
    gen = torch.Generator(device=device).manual_seed(7)
    bf = torch.bfloat16
    r = lambda *s: torch.randn(*s, generator=gen, device=device)
    pos = torch.randint(4096, 131072, (nseq,), generator=gen, device=device, dtype=torch.int64)
    ring_abs = pos[:, None] - W + torch.arange(W, device=device)[None]
    rp = torch.empty(nseq, W, dtype=torch.int64, device=device).scatter_(1, ring_abs % W, ring_abs)
    cache = dict(ring_k=r(nseq, G, W, D).to(bf), ring_v=r(nseq, G, W, D).to(bf), ring_km=r(nseq, W, G, D),
                 ring_g=r(nseq, W, G), ring_beta=r(nseq, W, G), ring_pos=rp, sink_k=r(nseq, G, S, D).to(bf),
                 sink_v=r(nseq, G, S, D).to(bf), S=r(nseq, G, D, D))
    n = llama_state_floats(G, D, W, S)
    rows = torch.empty(nseq, n, device=device)
    back = {k: torch.empty_like(v) for k, v in cache.items()}
    pack_ms = _time_device(lambda: pack_llama_state(L, cache, pos, rows=rows), steps, warmup)
    unpack_ms = _time_device(lambda: unpack_llama_state(L, rows, pos, cache=back), steps, warmup)
    ok = all(torch.equal(back[k], cache[k]) for k in cache)
    C = 3 * G * D + 2 * G
    cache_bytes = nseq * (2 * G * W * D * 2 + G * W * D * 4 + 2 * W * G * 4 + W * 8 + 2 * G * S * D * 2 + G * D * D * 4)
    pack_bytes = cache_bytes + nseq * n * 4
    unpack_bytes = cache_bytes + nseq * ((W + S) * C * 4 + G * D * D * 4)
    pk, _ = peaks()
    leg = lambda ms, nb: {"ms": ms, "bytes": nb, "achieved_gbs": nb / (ms * 1e-3) / 1e9,
                          "frac": nb / (ms * 1e-3) / 1e9 / pk["hbm_gbs"]}
    return {"workload": f"{nseq} sequences, W={W}, S={S}, G={G}, D={D}: one layer's decode cache <-> llama.cpp "
                        f"state rows ({n * 4 / 1e6:.1f} MB per sequence)",
            "pack": leg(pack_ms, pack_bytes), "unpack": leg(unpack_ms, unpack_bytes), "round_trip_exact": ok,
            "peak_gbs": pk["hbm_gbs"]}


# ---------------------------------------------------------------------------------------------- CPU arms
def cpu_sample_tokens_per_s(n_new=2048, start=None, seed=0, threads=None):
    """The CPU oracle (a restatement of the reference's PyTorch path, in the reference's own form: the prefill
    memory repeats the state for each query head, heimdall/hibrit.py:404-408) on a bounded sample of the
    workload: the last n_new tokens of the T=32768 prefill (positions start.. with a full synthetic cache: W
    ring entries, sinks, state), i.e. its steady-state per-token cost."""
    import torch.nn.functional as F
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    from oracle import bifrost_oracle as ob
    start = 32768 - n_new if start is None else start
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(seed)
    p = ob.init_params(H, G, D, DM, W, S, 1, "long", gen)
    n = lambda *s: torch.randn(*s, generator=gen)
    p.mix_w, p.mix_b, p.mix_lse, p.mem_scale = n(H, DM) * 0.02, n(H) * 0.02, n(H) * 0.02, n(H) * 0.02
    bfr = lambda z: z.to(torch.bfloat16).float()
    rms_ = lambda z: z * torch.rsqrt(z.square().mean(-1, keepdim=True) + 1e-6)
    x = bfr(n(1, n_new, DM))
    q, k, v = bfr(rms_(n(1, n_new, H, D))), bfr(rms_(n(1, n_new, G, D))), bfr(rms_(n(1, n_new, G, D)))
    qr, kr = bfr(rms_(n(1, H, n_new, D))), bfr(rms_(n(1, G, n_new, D)))
    pp = torch.arange(start - W, start)
    cache = dict(ring_k=bfr(rms_(n(1, G, W, D))), ring_v=bfr(rms_(n(1, G, W, D))),
                 ring_km=F.normalize(n(1, W, G, D), dim=-1), ring_g=-torch.rand(1, W, G, generator=gen) * 0.01,
                 ring_beta=torch.rand(1, W, G, generator=gen), ring_pos=torch.empty(W, dtype=torch.long),
                 sink_k=bfr(rms_(n(1, G, S, D))), sink_v=bfr(rms_(n(1, G, S, D))), S=n(1, G, D, D) * 0.02)
    cache["ring_pos"][pp % W] = pp
    t0 = time.perf_counter()
    with torch.no_grad():
        ob.student(p, x, q, k, v, qr, kr, start, cache, gqa_native=False)
    dt = time.perf_counter() - t0
    return n_new / dt, threads, dt


def cpu_baseline(min_seconds=10.0, n_new=2048):
    """Repeats the bounded sample until at least ``min_seconds`` of CPU work ran; tokens / total time."""
    tot_t, tot_n, reps = 0.0, 0, 0
    cores = 1
    while tot_t < min_seconds or reps < 2:
        _, cores, dt = cpu_sample_tokens_per_s(n_new)
        tot_t += dt
        tot_n += n_new
        reps += 1
    return tot_n / tot_t, cores, tot_t, reps


HEADLINE_T = 131072


def _set_headline(T: int) -> None:
    global HEADLINE_T
    HEADLINE_T = int(T)


def arm_config(world):
    return {"workload": f"BASELINE config 3 at T={HEADLINE_T}: one Bifrost layer prefill of one {HEADLINE_T}-token "
                        f"sequence (B=1, 24q/4kv heads, D=256, W=2048, 4 sinks, d=5120, from an empty cache) split "
                        f"evenly over the {world} GPU(s) (sequence-parallel; one GPU: an ordinary prefill)",
            "global_batch": 1, "seq_len": HEADLINE_T,
            "parallelism": f"sequence-parallel sp{world}" if world > 1 else "single GPU",
            "l2": "inputs larger than L2 (5.4 GB read per step on one GPU), no flush"}


def cpu_model():
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args, rank):
    """The reference's CPU path on the host cores: the oracle port in the reference's own form (the reference is
    PyTorch, nothing compiles into oracle/_ref; the port repeats the prefill state for each query head as
    heimdall/hibrit.py:404-408 does), all host threads, no GPU and no process group.  Each step is a bounded
    sample of the workload: the last n_new tokens of a long prefill against a full cache (W ring entries, sinks,
    state), whose per-token cost is the steady state of any prefill longer than 2W (32K and 128K alike); n_new
    shrinks for long runs so the whole --steps/--warmup run stays within a few minutes.  Under torchrun only
    rank 0 runs and prints."""
    if rank != 0:
        return
    n_new = 2048 if args.steps + args.warmup <= 150 else (1024 if args.steps + args.warmup <= 300 else 512)
    for _ in range(args.warmup):
        cpu_sample_tokens_per_s(n_new)
    tot = 0.0
    cores = 1
    for _ in range(args.steps):
        _, cores, dt = cpu_sample_tokens_per_s(n_new)
        tot += dt
    val = n_new * args.steps / tot
    sample = (f"{n_new} tokens per step: the last {n_new} tokens of a long prefill (positions from 32768 - {n_new}) "
              f"with a full cache (W=2048 ring, 4 sinks, state): the steady-state per-token cost of the prefill; "
              f"{cores} threads on {cpu_model()}")
    cfg = arm_config(args.gpus)
    cfg["sample"] = sample
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": val, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": tot / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, config-1/3 shapes)", "config": cfg,
        "cpu_baseline": {"value": val, "unit": "tok/s", "cores": cores, "cpu": cpu_model(), "kind": "port",
                         "form": "reference (state repeated per query head, hibrit.py:404-408)", "sample": sample},
        "e2e": {"value": val, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}), flush=True)


# ---------------------------------------------------------------------------------------------- driver
def barrier(ctx):
    if ctx["world"] > 1:
        torch.distributed.barrier()


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        # the sequence-parallel exchange runs beside the window kernel's queued CTAs: a high-priority NCCL
        # stream gets its CTAs dispatched first
        opts = torch.distributed.ProcessGroupNCCL.Options(is_high_priority_stream=True)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local), pg_options=opts)
    return {"world": world, "rank": rank, "local": local}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--T", type=int, default=32768, help="config-1 sequence length")
    ap.add_argument("--headline-T", type=int, default=HEADLINE_T,
                    help="headline sequence length (default 131072; smaller only for profiling captures)")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--decode-seqs", type=int, default=64)
    ap.add_argument("--decode-layers", type=int, default=12)
    ap.add_argument("--decode-steps", type=int, default=256)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-sp", action="store_true", help="skip the 1M-token sequence-parallel leg")
    ap.add_argument("--no-delta", action="store_true")
    ap.add_argument("--no-config1", action="store_true")
    ap.add_argument("--no-interchange", action="store_true", help="skip the llama.cpp state-row leg")
    ap.add_argument("--no-retrieval", action="store_true", help="skip the kept layers' retrieval decode leg")
    ap.add_argument("--no-backward", action="store_true", help="skip the delta-rule backward leg")
    args = ap.parse_args(argv)
    args.warmup = max(3, args.warmup)
    _set_headline(args.headline_T)
    if args.impl == "reference":
        # the CPU arm touches no GPU and joins no process group: rank 0 runs, the others leave
        run_reference(args, int(os.environ.get("RANK", "0")))
        return
    ctx = dist_setup()
    try:
        run_ours(args, ctx)
    finally:
        if ctx["world"] > 1 and torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()


def pick_peak(pk, clocks):
    """The bf16 peak that matches the timed region's clocks: the burst figure when the SMs ran at their maximum
    clock (median within 5 %), the sustained (power-capped) one otherwise."""
    med, mx = clocks.get("sm_mhz"), clocks.get("sm_max_mhz")
    if med and mx and med >= 0.95 * mx:
        return pk["bf16_tflops"], "burst"
    return pk["bf16_tflops_sustained"], "sustained"


def headline_flops(T_total):
    win_f, delta_f, proj_f = layer_flops(T_total)
    return win_f + delta_f + proj_f


def run_config1(L, dev, ctx, args, pk, pk_kind):
    """BASELINE config 1 on each GPU (a T=32768 layer prefill from an empty cache): stage times, the dominant
    kernel's roofline (the window, timed live on its stream), the layer roofline against the peak matching the
    clocks, and the window kernel alone."""
    T = args.T
    inputs = make_inputs(T, seed=1 + ctx["rank"], device=dev)
    stage_names = ["x_proj", "head_proj", "gdn_p1", "gdn_p2", "gdn_p3", "window_prep", "window", "cache"]
    steps = max(10, args.steps)
    with ClockSampler(ctx["local"]) as clk:
        ms, stage_ms = run_prefill(L, inputs, steps, args.warmup, T, ctx, stage_names)
    clocks = clk.summary()
    win_alone_ms = window_standalone_ms(inputs)
    del inputs
    t = torch.tensor([ms], device=dev)
    if ctx["world"] > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms_step = float(t.item()) / steps
    peak, peak_kind = pick_peak(pk, clocks)
    win_f, delta_f, proj_f = layer_flops(T)
    total_f = win_f + delta_f + proj_f
    win_ms = stage_ms.get("window")
    traffic = None
    tp = ROOT / "profiles" / "roofline_traffic.json"
    if tp.exists():
        try:
            traffic = json.loads(tp.read_text()).get("window_prefill_kernel_bytes_per_launch")
        except Exception:
            traffic = None
    roof = None
    if win_ms:
        ach = win_f / (win_ms * 1e-3) / 1e12
        alone = win_f / (win_alone_ms * 1e-3) / 1e12
        roof = {"kernel": "window_prefill_kernel", "bound": "tensor", "achieved": ach, "peak": peak,
                "unit": "TFLOP/s", "frac": ach / peak, "traffic": traffic, "flops_per_launch": win_f,
                "ms_per_launch": win_ms,
                "note": "ms_per_launch is the window's stage time inside the timed config-1 step, where it runs beside "
                        "the memory chain on the same SMs; standalone is the same kernel alone (with its V^T staging)",
                "standalone": {"ms_per_launch": win_alone_ms, "achieved": alone, "frac": alone / peak},
                "peak_source": f"{pk_kind} bf16 {peak_kind} (MEASURED_PEAKS.json; clocks median "
                               f"{clocks.get('sm_mhz')} of {clocks.get('sm_max_mhz')} MHz)",
                "frac_vs_burst": ach / pk["bf16_tflops"], "frac_vs_sustained": ach / pk["bf16_tflops_sustained"]}
    ach_layer = total_f / (ms_step * 1e-3) / 1e12
    return {"workload": "BASELINE config 1: single Bifrost layer prefill, T=32768, B=1 per GPU, 24q/4kv heads, "
                        "D=256, W=2048, 4 sinks, d=5120, from an empty cache",
            "value": T * ctx["world"] / (ms_step / 1e3), "unit": "tok/s", "ms_per_step": ms_step, "steps": steps,
            "stage_ms": stage_ms, "clocks": clocks, "roofline": roof,
            "layer_roofline": {"flops_per_step": total_f, "achieved_tflops": ach_layer, "peak": peak,
                               "peak_kind": peak_kind, "frac": ach_layer / peak,
                               "frac_vs_burst": ach_layer / pk["bf16_tflops"],
                               "frac_vs_sustained": ach_layer / pk["bf16_tflops_sustained"],
                               "split_flops": {"window": win_f, "delta_rule": delta_f, "projections": proj_f}}}


def run_headline(L, dev, ctx, args):
    """The headline: one HEADLINE_T-token sequence, sequence-parallel over the N GPUs (N=1: one prefill), timed
    with CUDA events over exactly --steps steps after --warmup, max over ranks, with clocks sampled."""
    from heimdall_b200 import sp
    world, rank = ctx["world"], ctx["rank"]
    T = HEADLINE_T // world
    ins = make_inputs(T, seed=11 + rank, device=dev)
    gr = None
    if world > 1:   # the sequence-parallel step captured once (collectives included) and replayed
        gr = sp.StudentSPGraph(L, *ins, warmup=args.warmup)
        step = gr.replay
    else:
        step = lambda: L.student(*ins, 0, {})
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(ctx)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with ClockSampler(ctx["local"]) as clk:
        torch.cuda.synchronize()
        h0 = time.perf_counter()
        evs[0].record()
        for i in range(args.steps):
            step()
            evs[i + 1].record()
        h1 = time.perf_counter()
        torch.cuda.synchronize()
    clocks = clk.summary()
    per = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    t = torch.tensor([evs[0].elapsed_time(evs[-1]) / args.steps], device=dev)
    if world > 1:
        gr.check()
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    del ins, gr
    diag = {"step_ms_min": min(per), "step_ms_median": statistics.median(per), "step_ms_max": max(per),
            "host_enqueue_ms_per_step": (h1 - h0) * 1e3 / args.steps}
    return float(t.item()), clocks, diag


def run_e2e(L, dev, ctx, steps):
    """The headline workload through the public API from pinned host buffers, copies inside the timed region:
    one GPU: ``BifrostLayer.student_host`` (4096-token chunks on three streams, copies overlapped with the
    layer); N GPUs: each rank copies its segment in, runs ``sp.student_sp`` and copies its outputs back.  Max
    over ranks."""
    from heimdall_b200 import sp
    world, rank = ctx["world"], ctx["rank"]
    T = HEADLINE_T // world
    host = [t.cpu().pin_memory() for t in make_inputs(T, 31 + rank, dev)]
    o_host = torch.empty(1, T, H, D, dtype=torch.float32).pin_memory()
    bi = sum(h.numel() * h.element_size() for h in host) * world
    bo = o_host.numel() * o_host.element_size() * world
    if world == 1:
        def step():
            L.student_host(*host, 0, None, out=o_host)
        api = "BifrostLayer.student_host (4096-token chunks, copies overlapped on three streams)"
    else:
        dbuf = [torch.empty_like(h, device=dev) for h in host]

        def step():
            for d_, h_ in zip(dbuf, host):
                d_.copy_(h_, non_blocking=True)
            o, _ = sp.student_sp(L, *dbuf)
            o_host.copy_(o, non_blocking=True)
            torch.cuda.current_stream().synchronize()
        api = "per rank: segment copied in, heimdall_b200.sp.student_sp, outputs copied back"
    step()
    torch.cuda.synchronize()
    barrier(ctx)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        step()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / steps], device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    return {"value": HEADLINE_T / (ms / 1e3), "unit": "tok/s", "ms_per_step": ms, "h2d_bytes_per_step": bi,
            "d2h_bytes_per_step": bo, "api": api, "steps": steps}


def run_ours(args, ctx):
    dev = torch.device("cuda", ctx["local"])
    torch.cuda.set_device(dev)
    world, rank = ctx["world"], ctx["rank"]
    L = make_layer(dev)
    pk, pk_kind = peaks()
    ms_step, clocks, diag = run_headline(L, dev, ctx, args)
    value = HEADLINE_T / (ms_step / 1e3)
    c1 = None if args.no_config1 else run_config1(L, dev, ctx, args, pk, pk_kind)
    e2e = None if args.no_e2e else run_e2e(L, dev, ctx, min(args.steps, 10))
    sp_131k = run_sp(L, dev, ctx, HEADLINE_T) if world > 1 else None
    sp_1m = None if args.no_sp else run_sp(L, dev, ctx, 1048576, steps=3, warmup=2)
    decode = None if args.no_decode else run_decode(dev, ctx, steps=args.decode_steps, nseq=args.decode_seqs,
                                                    nlayers=args.decode_layers)
    if rank != 0:
        return
    peak, peak_kind = pick_peak(pk, clocks)
    total_f = headline_flops(HEADLINE_T)
    ach = total_f / (ms_step * 1e-3) / 1e12
    # our kernels per step: x_proj, head_proj, P1, P2, V^T prep, window, P3 on one GPU; with N ranks the
    # worst rank adds the halo's two projections, the extended-key prep, the prefix fold and the second scan
    launches = 7 if world == 1 else 12
    out = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
           "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded; config-1/3 shapes and distributions)",
           "config": arm_config(world), "clocks": clocks, "step_diag_rank0": diag,
           "layer_roofline": {"flops_per_step": total_f, "achieved_tflops": ach, "peak": peak, "peak_kind": peak_kind,
                              "frac": ach / peak / world, "frac_vs_burst": ach / pk["bf16_tflops"] / world,
                              "frac_vs_sustained": ach / pk["bf16_tflops_sustained"] / world,
                              "note": "all algorithmic FLOPs of the step over N x the measured peak"},
           "gpu_launches": launches * args.steps}
    if c1 is not None:
        out["roofline"] = c1["roofline"]
        out["config1"] = c1
    if e2e is not None:
        out["e2e"] = e2e
    if sp_131k is not None:
        out["sp_131k"] = sp_131k
    if sp_1m is not None:
        out["sp_1m"] = sp_1m
    if not args.no_cpu and world == 1:
        tps, cores, dt, reps = cpu_baseline()
        out["cpu_baseline"] = {"value": tps, "unit": "tok/s", "cores": cores, "cpu": cpu_model(), "kind": "port",
                               "form": "reference (state repeated per query head, hibrit.py:404-408)",
                               "sample": f"{reps} x the last 2048 tokens of a long prefill against a full cache "
                                         f"(its steady-state per-token cost), {dt:.1f} s on {cores} threads"}
    if world == 1 and not args.no_delta:
        out["delta_rule"] = run_delta_configs(dev)
    if decode is not None:
        out["decode"] = decode
    if world == 1 and not args.no_interchange:
        out["interchange"] = run_interchange(dev)
    if world == 1 and not args.no_retrieval:
        out["retrieval"] = run_retrieval(dev)
    if world == 1 and not args.no_backward:
        out["backward"] = run_backward(dev)
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()

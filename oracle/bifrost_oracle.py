"""CPU oracle for the Bifrost converted-layer hot path.  TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The CUDA path in ``heimdall_b200`` never
calls into it and has no CPU fallback.

It restates, in plain PyTorch on the CPU, the arithmetic of Heimdall's Bifrost
layer (reference project ``Heimdall``, package ``heimdall``):

* ``gdn_chunked``   -- chunked gated delta rule, UT/WY form
                       (``heimdall/kernels.py:80-129``: ``_unit_lower_inverse``,
                       ``delta_rule_reference``)
* ``gdn_step``      -- one recurrent token (``heimdall/kernels.py:132-138``)
* ``gdn_recurrent`` -- the token loop over ``gdn_step`` (the recurrent form the
                       chunked one is tested against, ``tests/test_heimdall.py:36-48``)
* ``gdn_gqa``       -- one state per KV head read by R query heads
                       (``heimdall/motor.py:70-102``)
* ``window_attention`` -- sliding window plus sinks, fp32, with log-sum-exp
                       (``heimdall/hibrit.py:336-361``)
* ``mem_inputs``    -- memory read/write vectors, decay and write strength
                       (``heimdall/hibrit.py:327-334``)
* ``student``       -- the whole layer core with the reference's cache dict
                       (``heimdall/hibrit.py:363-424``)
* ``init_params``   -- the conversion-time parameter init
                       (``heimdall/hibrit.py:211-240``)
* ``proj`` / ``out`` / ``attention_forward`` -- the layer around the core:
                       projections, ZNorm and partial RoPE, the output gate and
                       o_proj (``heimdall/hibrit.py:246-272, 426-432``;
                       ``heimdall/kernels.py:40-49``)

Parity of this restatement is pinned against the reference itself: the fixtures
in ``tests/golden/`` were produced by importing the reference and running it on
seeded inputs (``tests/golden/make_golden.py``), and ``tests/test_oracle.py``
checks every function here against them.

Every function takes ``dtype`` (default float32, like the reference); float64
gives a higher-precision "truth" for error budgets.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.nn.functional as F


# --------------------------------------------------------------------------- parameters
@dataclass
class LayerParams:
    """The trained per-layer tensors of a converted layer (``heimdall/hibrit.py:196, 211-240``).

    Shapes: fq [H,D,D], fk [G,D,D], ab_w [2G,d], ab_b [2G], mix_w [H,d], mix_b [H],
    mix_lse [H], mem_scale [H], A_log [G], dt_bias [G], decay_mask [G] (0 = archival head).
    """
    fq: torch.Tensor
    fk: torch.Tensor
    ab_w: torch.Tensor
    ab_b: torch.Tensor
    mix_w: torch.Tensor
    mix_b: torch.Tensor
    mix_lse: torch.Tensor
    mem_scale: torch.Tensor
    A_log: torch.Tensor
    dt_bias: torch.Tensor
    decay_mask: torch.Tensor
    window: int
    sinks: int
    extra: dict = field(default_factory=dict)

    @property
    def n_heads(self) -> int:
        return self.fq.shape[0]

    @property
    def n_kv(self) -> int:
        return self.fk.shape[0]

    @property
    def head_dim(self) -> int:
        return self.fq.shape[-1]

    def to(self, device=None, dtype=None) -> "LayerParams":
        conv = lambda t: t.to(device=device, dtype=dtype if t.is_floating_point() else None)
        kw = {k: conv(getattr(self, k)) for k in ("fq", "fk", "ab_w", "ab_b", "mix_w", "mix_b", "mix_lse",
                                                 "mem_scale", "A_log", "dt_bias", "decay_mask")}
        return LayerParams(window=self.window, sinks=self.sinks, extra=dict(self.extra), **kw)


def params_from_module(attn) -> LayerParams:
    """Read a converted reference ``HybridAttention`` into a ``LayerParams`` (fp32 copies)."""
    f = lambda t: t.detach().float().cpu().clone()
    return LayerParams(fq=f(attn.fq), fk=f(attn.fk), ab_w=f(attn.ab.weight), ab_b=f(attn.ab.bias),
                       mix_w=f(attn.mix.weight), mix_b=f(attn.mix.bias), mix_lse=f(attn.mix_lse),
                       mem_scale=f(attn.mem_scale), A_log=f(attn.A_log), dt_bias=f(attn.dt_bias),
                       decay_mask=f(attn.decay_mask), window=int(attn.window), sinks=int(attn.sinks))


def init_params(H: int, G: int, D: int, d: int, window: int, sinks: int, archival: int,
                mem_init: str = "long", generator: Optional[torch.Generator] = None) -> LayerParams:
    """Conversion-time init, restating ``HybridAttention.convert`` (``heimdall/hibrit.py:211-240``).

    fq/fk are identities, ab/mix are zero with mix bias -2, mix_lse is zero, dt is log-uniform in
    [1e-3, 1e-1] with dt_bias = softplus^-1(dt); "long" sets half-lives log-spaced from the window to
    1e6 tokens and mem_scale = sqrt(D); "mamba" sets A in U[1,16] and mem_scale = 1.  The first
    ``archival`` KV heads never decay (decay_mask 0).
    """
    gen = generator
    eye = torch.eye(D)
    dt = torch.exp(torch.empty(G).uniform_(math.log(1e-3), math.log(1e-1), generator=gen))
    dt_bias = dt + torch.log(-torch.expm1(-dt))
    if mem_init == "mamba":
        mem_scale = torch.ones(H)
        A_log = torch.empty(G).uniform_(1.0, 16.0, generator=gen).log()
    else:
        mem_scale = torch.full((H,), float(D) ** 0.5)
        life = torch.logspace(math.log10(max(window, 2)), 6.0, G)
        A_log = (math.log(2.0) / (life * dt)).log()
    mask = torch.ones(G)
    mask[:archival] = 0.0
    return LayerParams(fq=eye.repeat(H, 1, 1), fk=eye.repeat(G, 1, 1), ab_w=torch.zeros(2 * G, d),
                       ab_b=torch.zeros(2 * G), mix_w=torch.zeros(H, d), mix_b=torch.full((H,), -2.0),
                       mix_lse=torch.zeros(H), mem_scale=mem_scale, A_log=A_log, dt_bias=dt_bias,
                       decay_mask=mask, window=window, sinks=sinks)


# --------------------------------------------------------------------------- gated delta rule
def unit_lower_inverse(a: torch.Tensor) -> torch.Tensor:
    """(I + A)^-1 for strictly lower-triangular A (``heimdall/kernels.py:81-91``)."""
    n = a.shape[-1]
    eye = torch.eye(n, dtype=a.dtype)
    rhs = eye.expand(a.shape).contiguous()
    return torch.linalg.solve_triangular(eye + a, rhs, upper=False, unitriangular=True)


def gdn_chunked(q, k, v, g, beta, chunk: int = 64, s0=None, dtype=torch.float32):
    """Chunked gated delta rule, restating ``delta_rule_reference`` (``heimdall/kernels.py:94-129``).

    Recurrence: S_t = a_t S_{t-1} + beta_t k_t (v_t - a_t S_{t-1}^T k_t)^T, o_t = S_t^T q_t, a_t = e^{g_t}.
    q, k: [B,T,H,Dk]; v: [B,T,H,Dv]; g, beta: [B,T,H]; s0: [B,H,Dk,Dv] or None.
    Returns o [B,T,H,Dv] and the final state [B,H,Dk,Dv] in ``dtype``.

    Per chunk of C tokens (cumulative log-decay c_i = sum_{j<=i} g_j inside the chunk):
      L_ij = e^{c_i - c_j} (i >= j),  A = strict_lower(beta_i k_i.k_j L_ij),  Tm = (I + A)^-1,
      u = Tm (beta v),  w = Tm (beta e^{c} k),  P = (q k^T) * L  (lower incl. diagonal),
      v' = u - w S,  o = (e^{c} q) S + P v',  S <- e^{c_C} S + (e^{c_C - c} k)^T v'.
    Padding to a multiple of C uses g = beta = 0 rows, which leave S unchanged.
    """
    B, T, H, Dk = k.shape
    Dv = v.shape[-1]
    q, k, v, g, beta = (z.to(dtype) for z in (q, k, v, g, beta))
    C = chunk
    n = (T + C - 1) // C
    pad = n * C - T
    if pad:
        q = F.pad(q, (0, 0, 0, 0, 0, pad))
        k = F.pad(k, (0, 0, 0, 0, 0, pad))
        v = F.pad(v, (0, 0, 0, 0, 0, pad))
        g = F.pad(g, (0, 0, 0, pad))
        beta = F.pad(beta, (0, 0, 0, pad))
    # head-major chunk views [B,H,n,C,*]
    hm = lambda z: z.transpose(1, 2).reshape(B, H, n, C, *z.shape[3:])
    q, k, v, g, beta = hm(q), hm(k), hm(v), hm(g), hm(beta)
    S = torch.zeros(B, H, Dk, Dv, dtype=dtype) if s0 is None else s0.to(dtype).clone()
    out = torch.empty(B, H, n, C, Dv, dtype=dtype)
    tril = torch.ones(C, C, dtype=torch.bool).tril()
    for c in range(n):
        kc, vc, qc, bc = k[:, :, c], v[:, :, c], q[:, :, c], beta[:, :, c]
        cum = g[:, :, c].cumsum(-1)                                       # [B,H,C]
        L = torch.where(tril, (cum[..., :, None] - cum[..., None, :]).masked_fill(~tril, 0).exp(),
                        torch.zeros((), dtype=dtype))
        kb = kc * bc[..., None]
        A = ((kb @ kc.transpose(-1, -2)) * L).tril(-1)
        Tm = unit_lower_inverse(A)
        u = Tm @ (vc * bc[..., None])
        w = Tm @ (kb * cum.exp()[..., None])
        P = (qc @ kc.transpose(-1, -2)) * L
        vnew = u - w @ S
        out[:, :, c] = (qc * cum.exp()[..., None]) @ S + P @ vnew
        tail = (cum[..., -1:] - cum).exp()[..., None]                      # [B,H,C,1]
        S = S * cum[..., -1].exp()[..., None, None] + (kc * tail).transpose(-1, -2) @ vnew
    o = out.reshape(B, H, n * C, Dv)[:, :, :T].transpose(1, 2)
    return o, S


def gdn_step(q, k, v, g, beta, state, dtype=torch.float32):
    """One recurrent token, restating ``delta_rule_step`` (``heimdall/kernels.py:132-138``).

    q, k: [B,H,Dk]; v: [B,H,Dv]; g, beta: [B,H]; state [B,H,Dk,Dv].  Returns (o [B,H,Dv], new state).
    """
    q, k, v, g, beta, S = (z.to(dtype) for z in (q, k, v, g, beta, state))
    S = S * g.exp()[..., None, None]
    err = v - (k[..., :, None] * S).sum(-2)
    S = S + k[..., :, None] * (err * beta[..., None])[..., None, :]
    return (q[..., :, None] * S).sum(-2), S


def gdn_recurrent(q, k, v, g, beta, s0=None, dtype=torch.float32):
    """Token-by-token form of the same recurrence (``gdn_step`` in a loop); [B,T,H,*] layouts."""
    B, T, H, Dk = k.shape
    Dv = v.shape[-1]
    S = torch.zeros(B, H, Dk, Dv, dtype=dtype) if s0 is None else s0.to(dtype)
    outs = []
    for t in range(T):
        o, S = gdn_step(q[:, t], k[:, t], v[:, t], g[:, t], beta[:, t], S, dtype)
        outs.append(o)
    return torch.stack(outs, 1), S


def gdn_gqa(q, k, v, g, beta, chunk: int = 64, state=None, dtype=torch.float32):
    """GQA-native gated delta rule, restating ``delta_rule_gqa`` (``heimdall/motor.py:70-102``).

    q [B,T,G,R,Dk]; k [B,T,G,Dk]; v [B,T,G,Dv]; g, beta [B,T,G]; state [B,G,Dk,Dv].
    Returns o [B,T,G,R,Dv] and the final state [B,G,Dk,Dv].  The state is written once per KV head
    and read by the R query heads of its group; the arithmetic is ``gdn_chunked`` with the R query
    heads stacked along the row dimension of the read.
    """
    B, T, G, R, Dk = q.shape
    Dv = v.shape[-1]
    q, k, v, g, beta = (z.to(dtype) for z in (q, k, v, g, beta))
    C = chunk
    n = (T + C - 1) // C
    pad = n * C - T
    if pad:
        q = F.pad(q, (0, 0, 0, 0, 0, 0, 0, pad))
        k = F.pad(k, (0, 0, 0, 0, 0, pad))
        v = F.pad(v, (0, 0, 0, 0, 0, pad))
        g = F.pad(g, (0, 0, 0, pad))
        beta = F.pad(beta, (0, 0, 0, pad))
    qh = q.permute(0, 2, 3, 1, 4).reshape(B, G, R, n, C, Dk)
    hm = lambda z: z.transpose(1, 2).reshape(B, G, n, C, *z.shape[3:])
    k, v, g, beta = hm(k), hm(v), hm(g), hm(beta)
    S = torch.zeros(B, G, Dk, Dv, dtype=dtype) if state is None else state.to(dtype).clone()
    out = torch.empty(B, G, R, n, C, Dv, dtype=dtype)
    tril = torch.ones(C, C, dtype=torch.bool).tril()
    for c in range(n):
        kc, vc, bc = k[:, :, c], v[:, :, c], beta[:, :, c]
        qc = qh[:, :, :, c]                                               # [B,G,R,C,Dk]
        cum = g[:, :, c].cumsum(-1)
        L = torch.where(tril, (cum[..., :, None] - cum[..., None, :]).masked_fill(~tril, 0).exp(),
                        torch.zeros((), dtype=dtype))
        kb = kc * bc[..., None]
        Tm = unit_lower_inverse(((kb @ kc.transpose(-1, -2)) * L).tril(-1))
        u = Tm @ (vc * bc[..., None])
        w = Tm @ (kb * cum.exp()[..., None])
        vnew = u - w @ S                                                  # [B,G,C,Dv]
        P = (qc @ kc[:, :, None].transpose(-1, -2)) * L[:, :, None]       # [B,G,R,C,C]
        out[:, :, :, c] = (qc * cum.exp()[:, :, None, :, None]) @ S[:, :, None] + P @ vnew[:, :, None]
        tail = (cum[..., -1:] - cum).exp()[..., None]
        S = S * cum[..., -1].exp()[..., None, None] + (kc * tail).transpose(-1, -2) @ vnew
    o = out.reshape(B, G, R, n * C, Dv)[:, :, :, :T].permute(0, 3, 1, 2, 4)
    return o, S


# --------------------------------------------------------------------------- window attention
def window_attention(qr, ext_k, ext_v, ext_pos, sink_k, sink_v, pos, window: int, sinks: int,
                     dtype=torch.float32, block: int = 0):
    """Sliding-window + sink attention with log-sum-exp, restating ``_window_fp32`` (``heimdall/hibrit.py:341-361``).

    qr [B,H,t,D] (RoPE applied); ext_k/ext_v [B,G,W+t,D] (ring in time order, then the new tokens);
    ext_pos [W+t] (-1 = empty slot); sink_k/sink_v [B,G,ns,D] or None (positions 0..ns-1); pos [t].
    A query at position p sees key position kp when kp >= 0, kp <= p and either kp is a sink or
    (p - kp < window and kp >= sinks).  Scores use q * D^-1/2.
    Returns o [B,t,H,D] and lse [B,H,t] in ``dtype``.
    """
    B, H, t, D = qr.shape
    G = ext_k.shape[1]
    R = H // G
    q = qr.to(dtype).reshape(B, G, R, t, D) * D ** -0.5
    ns = 0 if sink_k is None else sink_k.shape[2]
    blk = block or max(window, 1)
    o = torch.empty(B, G, R, t, D, dtype=dtype)
    lse = torch.empty(B, G, R, t, dtype=dtype)
    for q0 in range(0, t, blk):
        q1 = min(t, q0 + blk)
        # query i (absolute row q0+i) can only see ext rows [q0, q1 + window)
        e0, e1 = q0, min(ext_k.shape[2], q1 + window)
        keys, vals, kpos = ext_k[:, :, e0:e1].to(dtype), ext_v[:, :, e0:e1].to(dtype), ext_pos[e0:e1]
        sink = torch.zeros(e1 - e0, dtype=torch.bool)
        if ns:
            keys = torch.cat((sink_k.to(dtype), keys), 2)
            vals = torch.cat((sink_v.to(dtype), vals), 2)
            kpos = torch.cat((torch.arange(ns, dtype=kpos.dtype), kpos))
            sink = torch.cat((torch.ones(ns, dtype=torch.bool), sink))
        qp = pos[q0:q1, None]
        ok = (kpos[None] >= 0) & (kpos[None] <= qp) & (sink[None] | ((qp - kpos[None] < window) & (kpos[None] >= sinks)))
        sc = torch.einsum("bgrqd,bgkd->bgrqk", q[:, :, :, q0:q1], keys)
        sc = sc.masked_fill(~ok, float("-inf"))
        m = sc.logsumexp(-1)
        o[:, :, :, q0:q1] = torch.einsum("bgrqk,bgkd->bgrqd", (sc - m[..., None]).exp(), vals)
        lse[:, :, :, q0:q1] = m
    return o.reshape(B, H, t, D).transpose(1, 2), lse.reshape(B, H, t)


# --------------------------------------------------------------------------- memory inputs, gate, layer
def mem_inputs(p: LayerParams, x, q, k, pos, dtype=torch.float32):
    """Memory vectors and gates, restating ``_mem_inputs`` (``heimdall/hibrit.py:327-334``).

    qm = unit(q_h fq_h) D^-1/2, km = unit(k_g fk_g) (unit = F.normalize, eps 1e-12),
    [a | b] = x ab_w^T + ab_b, g = -e^{A_log} softplus(a + dt_bias) * decay_mask,
    beta = sigmoid(b) * [pos >= sinks].
    x [B,t,d], q [B,t,H,D], k [B,t,G,D], pos [t] -> qm [B,t,H,D], km [B,t,G,D], g, beta [B,t,G].
    """
    D = q.shape[-1]
    G = k.shape[2]
    qm = F.normalize(torch.einsum("bthd,hde->bthe", q.to(dtype), p.fq.to(dtype)), dim=-1) * D ** -0.5
    km = F.normalize(torch.einsum("bthd,hde->bthe", k.to(dtype), p.fk.to(dtype)), dim=-1)
    ab = x.to(dtype) @ p.ab_w.to(dtype).t() + p.ab_b.to(dtype)
    a, b = ab[..., :G], ab[..., G:]
    g = -p.A_log.to(dtype).exp() * F.softplus(a + p.dt_bias.to(dtype)) * p.decay_mask.to(dtype)
    beta = torch.sigmoid(b) * (pos >= p.sinks).to(dtype)[None, :, None]
    return qm, km, g, beta


def gate(p: LayerParams, x, lse, pos, dtype=torch.float32):
    """gamma = sigmoid(x mix_w^T + mix_b + mix_lse (lse - ln W)) * [pos >= W]  (``heimdall/hibrit.py:409-410``).

    x [B,t,d], lse [B,H,t] -> gamma [B,t,H].
    """
    z = x.to(dtype) @ p.mix_w.to(dtype).t() + p.mix_b.to(dtype)
    z = z + p.mix_lse.to(dtype) * (lse.to(dtype).transpose(1, 2) - math.log(p.window))
    return torch.sigmoid(z) * (pos >= p.window).to(dtype)[None, :, None]


def mix(p: LayerParams, o_win, o_mem, gamma, dtype=torch.float32):
    """o = o_win + gamma (mem_scale o_mem - o_win)  (``heimdall/hibrit.py:411``); [B,t,H,D]."""
    return o_win + gamma[..., None] * (p.mem_scale.to(dtype)[:, None] * o_mem - o_win)


def student(p: LayerParams, x, q, k, v, qr, kr, start: int, cache: Optional[dict], memory: bool = True,
            dtype=torch.float32, gqa_native: bool = True):
    """The converted layer core, restating ``HybridAttention._student`` (``heimdall/hibrit.py:363-424``).

    x [B,t,d]; q [B,t,H,D] (pre-RoPE); k, v [B,t,G,D]; qr [B,H,t,D]; kr [B,G,t,D]; ``start`` is the
    absolute position of the first token.  ``cache`` (or None) is the reference's per-layer dict,
    updated in place with keys ring_k, ring_v [B,G,W,D] (kr/v dtype), ring_km [B,W,G,D], ring_g,
    ring_beta [B,W,G], ring_pos [W] (int64, -1 = empty), sink_k, sink_v [B,G,<=S,D] and S [B,G,D,D].
    Memory writes are delayed by W: the write stream at step i is token i - W (from the ring for the
    first W rows, then the new tokens), so a token enters memory exactly when it leaves the window.
    Returns o [B,t,H,D] in ``dtype``.

    ``gqa_native`` (default) runs the memory of a prefill with one state per KV head read by its R query heads
    (``gdn_gqa``, the arithmetic of ``heimdall/motor.py:70-102``).  ``gqa_native=False`` follows the reference's
    own ``_student`` statement for statement instead: for t > 1 the write stream and the state are repeated for
    every query head and ``gdn_chunked`` runs over H heads, then every R-th state is kept
    (``heimdall/hibrit.py:404-408``); for t == 1 the inline update (``:398-403``).  Both give the same
    numbers (the reference's own check, ``tests/test_motor.py:28-39``); the second does the reference's amount
    of work (R times the state traffic), which is what the timed CPU baseline runs.
    """
    B, t, _ = x.shape
    H, G, D = q.shape[2], k.shape[2], q.shape[3]
    W, S_, R = p.window, p.sinks, H // G
    st = cache if cache is not None else {}
    pos = torch.arange(start, start + t)
    vt = v.transpose(1, 2)
    sink_k, sink_v = st.get("sink_k"), st.get("sink_v")
    n_new = max(0, min(t, S_ - start))
    if n_new:
        nk, nv = kr[:, :, :n_new], vt[:, :, :n_new]
        sink_k = nk if sink_k is None else torch.cat((sink_k, nk), 2)
        sink_v = nv if sink_v is None else torch.cat((sink_v, nv), 2)
    ring_pos_expected = torch.arange(start - W, start)
    if "ring_k" in st:
        slots = ring_pos_expected % W
        rk, rv = st["ring_k"][:, :, slots], st["ring_v"][:, :, slots]
        rkm, rg, rb = st["ring_km"][:, slots], st["ring_g"][:, slots], st["ring_beta"][:, slots]
        valid = st["ring_pos"][slots] == ring_pos_expected
    else:
        rk, rv = kr.new_zeros(B, G, W, D), vt.new_zeros(B, G, W, D)
        rkm = torch.zeros(B, W, G, D)
        rg, rb = torch.zeros(B, W, G), torch.zeros(B, W, G)
        valid = torch.zeros(W, dtype=torch.bool)
    ext_pos = torch.cat((torch.where(valid, ring_pos_expected, torch.full_like(ring_pos_expected, -1)), pos))
    ext_k = torch.cat((rk.to(kr.dtype), kr), 2)
    ext_v = torch.cat((rv.to(vt.dtype), vt), 2)
    o_win, lse = window_attention(qr, ext_k, ext_v, ext_pos, sink_k, sink_v, pos, W, S_, dtype)
    o = o_win
    use_mem = memory and start + t > W
    if use_mem or cache is not None:
        qm, km, g, beta = mem_inputs(p, x, q, k, pos, dtype)
    if use_mem:
        vf = valid.to(dtype)[None, :, None]
        wk = torch.cat((rkm.to(dtype), km), 1)[:, :t]
        wv = torch.cat((rv.transpose(1, 2).to(dtype), v.to(dtype)), 1)[:, :t]
        wg = torch.cat((rg.to(dtype) * vf, g), 1)[:, :t]
        wb = torch.cat((rb.to(dtype) * vf, beta), 1)[:, :t]
        s0 = st.get("S")
        if gqa_native or t == 1:
            o_mem, Snew = gdn_gqa(qm.reshape(B, t, G, R, D), wk, wv, wg, wb, 64, s0, dtype)
        else:
            rep = lambda z: z.repeat_interleave(R, 2)
            o_mem, Snew = gdn_chunked(qm, rep(wk), rep(wv), rep(wg), rep(wb), 64,
                                      None if s0 is None else s0.repeat_interleave(R, 1), dtype)
            Snew = Snew[:, ::R]
        o_mem = o_mem.reshape(B, t, H, D)
        gm = gate(p, x, lse, pos, dtype)
        o = mix(p, o_win, o_mem, gm, dtype)
        if cache is not None:
            cache["S"] = Snew.float()
    if cache is not None:
        if "ring_k" not in cache:
            cache.update(ring_k=rk, ring_v=rv, ring_km=rkm, ring_g=rg, ring_beta=rb,
                         ring_pos=torch.full((W,), -1, dtype=torch.long))
        m = min(t, W)
        slot = pos[-m:] % W
        cache["ring_k"][:, :, slot] = kr[:, :, -m:].to(cache["ring_k"].dtype)
        cache["ring_v"][:, :, slot] = vt[:, :, -m:].to(cache["ring_v"].dtype)
        cache["ring_km"][:, slot] = km[:, -m:].float()
        cache["ring_g"][:, slot] = g[:, -m:].float()
        cache["ring_beta"][:, slot] = beta[:, -m:].float()
        cache["ring_pos"][slot] = pos[-m:]
        cache["sink_k"], cache["sink_v"] = sink_k, sink_v
    return o


# --------------------------------------------------------------------------- the layer around the core
@dataclass
class ProjParams:
    """The converted layer's frozen projections (``HybridAttention.__init__``, ``heimdall/hibrit.py:199-209``):
    q_w [H*D*(2 if gated), d] (query and output gate interleaved per head), k_w, v_w [G*D, d], o_w [d, H*D],
    optional biases, q_norm_w / k_norm_w [D] (ZNorm weights, zero-centred), rotary dims ``rot`` and base
    ``theta``, ``eps``."""
    q_w: torch.Tensor
    k_w: torch.Tensor
    v_w: torch.Tensor
    o_w: torch.Tensor
    q_norm_w: torch.Tensor
    k_norm_w: torch.Tensor
    rot: int
    theta: float
    eps: float = 1e-6
    gated: bool = True
    q_b: Optional[torch.Tensor] = None
    k_b: Optional[torch.Tensor] = None
    v_b: Optional[torch.Tensor] = None
    o_b: Optional[torch.Tensor] = None


def znorm(x, w, eps):
    """Qwen3.5 RMSNorm with a zero-centred weight, ``ZNorm.forward`` (``heimdall/hibrit.py:105-116``):
    x * rsqrt(mean(x^2) + eps) * (1 + w) in fp32, returned in x's dtype."""
    xf = x.float()
    return (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps) * (1.0 + w.float())).to(x.dtype)


def rope_inv_freq(d: int, base: float) -> torch.Tensor:
    """Inverse frequencies of ``kernels.rope`` (``heimdall/kernels.py:40-49``), fp32: 1 / base^(2i/d)."""
    return 1.0 / (base ** (torch.arange(0, d, 2, dtype=torch.float32) / d))


def rope(x, pos, base: float):
    """Half-rotation RoPE, restating ``kernels.rope`` (``heimdall/kernels.py:40-49``): x [B,H,T,d] and positions
    [T]; (x1, x2) = halves of the last dim, out = (x1 cos - x2 sin, x1 sin + x2 cos), computed in fp32 and
    returned in x's dtype."""
    d = x.shape[-1]
    ang = pos.to(torch.float32)[..., None] * rope_inv_freq(d, base)
    cos, sin = ang.cos(), ang.sin()
    x1, x2 = x.float().chunk(2, dim=-1)
    return torch.cat((x1 * cos - x2 * sin, x1 * sin + x2 * cos), dim=-1).to(x.dtype)


def partial_rope(x, pos, rot: int, base: float):
    """``HybridAttention._rope`` (``heimdall/hibrit.py:246-252``): RoPE on the first ``rot`` dims only."""
    if rot == 0:
        return x
    if rot == x.shape[-1]:
        return rope(x, pos, base)
    return torch.cat((rope(x[..., :rot], pos, base), x[..., rot:]), dim=-1)


def proj(pp: ProjParams, x, start: int):
    """``HybridAttention._proj`` (``heimdall/hibrit.py:254-268``): x [B,t,d] (bf16) -> q [B,t,H,D], k, v
    [B,t,G,D], qr [B,H,t,D], kr [B,G,t,D] (ZNorm'd, partial RoPE) and the output gate [B,t,H*D] (or None),
    all in x's dtype (the projections run in x's dtype, as the reference's bf16 Linear layers do)."""
    B, t, _ = x.shape
    D = pp.q_norm_w.shape[0]
    G = pp.k_w.shape[0] // D
    qg = F.linear(x, pp.q_w.to(x.dtype), None if pp.q_b is None else pp.q_b.to(x.dtype))
    gate = None
    if pp.gated:
        H = qg.shape[-1] // (2 * D)
        q, gate = qg.view(B, t, H, 2 * D).chunk(2, dim=-1)
        gate = gate.reshape(B, t, H * D)
    else:
        H = qg.shape[-1] // D
        q = qg.view(B, t, H, D)
    q = znorm(q, pp.q_norm_w, pp.eps)
    k = znorm(F.linear(x, pp.k_w.to(x.dtype), None if pp.k_b is None else pp.k_b.to(x.dtype)).view(B, t, G, D),
              pp.k_norm_w, pp.eps)
    v = F.linear(x, pp.v_w.to(x.dtype), None if pp.v_b is None else pp.v_b.to(x.dtype)).view(B, t, G, D)
    pos = torch.arange(start, start + t)
    return (q, k, v, partial_rope(q.transpose(1, 2), pos, pp.rot, pp.theta),
            partial_rope(k.transpose(1, 2), pos, pp.rot, pp.theta), gate)


def out(pp: ProjParams, o, gate, x):
    """``HybridAttention._out`` (``heimdall/hibrit.py:270-272``): o [B,t,H,D] -> o_proj(o * sigmoid(gate)) in
    x's dtype."""
    o = o.reshape(*x.shape[:2], -1).to(x.dtype)
    if gate is not None:
        o = o * torch.sigmoid(gate)
    return F.linear(o, pp.o_w.to(x.dtype), None if pp.o_b is None else pp.o_b.to(x.dtype))


def attention_forward(p: LayerParams, pp: ProjParams, x, cache: Optional[dict], start: int = 0, memory: bool = True):
    """``HybridAttention.forward`` of a converted layer in student mode (``memory=False``: window mode)
    (``heimdall/hibrit.py:426-432``): _proj -> _student -> _out.  x [B,t,d] -> y [B,t,d] in x's dtype."""
    q, k, v, qr, kr, gate = proj(pp, x, start)
    o = student(p, x, q, k, v, qr, kr, start, cache, memory=memory)
    return out(pp, o, gate, x)


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    """||a - b|| / ||b|| in float64."""
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-300))

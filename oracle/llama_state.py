"""CPU oracle for the llama.cpp Bifrost state row.  TEST INFRASTRUCTURE ONLY.

This module is a checker, never the product: only ``tests/`` and ``bench.py``'s CPU legs may import it.  The
product's pack / unpack run in CUDA (``bf_llama_state_pack`` / ``bf_llama_state_unpack``) with no CPU fallback.

It restates the per-sequence state row that the reference's llama.cpp port keeps for every converted layer
(reference project ``Heimdall``, file ``llamacpp/bifrost.patch``), all fp32, ggml order (ne0 fastest):

* ``ring_channels``  -- C = 3 G D + 2 G channels of a region row [k_rope | v | k_mem | g | beta]
                        (``llama_hparams::bifrost_ring_ch``, bifrost.patch:221-224; row assembly :990-996)
* ``region_slots``   -- LR = round_up(S + W + 2, 32) slots: sinks | ring of W + 1 slots (slot = S + pos mod (W+1))
                        | scratch + padding (``bifrost_region``, :226-228; slot rule :848)
* ``state_floats``   -- LR (C + 2 G D) + D D G floats: region [C, LR], K plane [D, LR, G], transposed V plane
                        [LR, D, G], delta state [D, D, G] (``bifrost_state``, :230-239; offsets :1010-1013)
* ``pack`` / ``unpack`` -- between that row and the reference's cache dict (``heimdall/hibrit.py:414-423``)
* ``llama_decode``   -- one decode token of the port's graph over a row (:841-927 inputs and mask, :1040-1054
                        decode writes and attention, :1093-1166 lse, memory update and mix), so that a packed row
                        can be shown to continue a sequence exactly as the reference's ``_student`` continues the
                        cache it was packed from.

Orientation of the delta state: the decode reads the memory as ``ggml_mul_mat(s_new, qm)`` (bifrost.patch:1129),
which contracts over ne0, so ne0 is the key index: element (key k, value v) of KV head g sits at
``off_delta + (g D + v) D + k``, the transpose of the reference's ``S[b, g, k, v]``.

Positions are not stored in the row (llama.cpp keeps them in its memory cells), so ``unpack`` and ``llama_decode``
take the sequence's next position.  ``pack`` takes it too and writes a ring slot only when the cache's
``ring_pos`` holds the position that slot must hold; every slot that no future step reads (negative positions,
the stale (W+1)-th ring slot, scratch, padding, sink slots not yet reached) is zero.
"""
from __future__ import annotations

import math

import torch


def ring_channels(G: int, D: int) -> int:
    return 3 * G * D + 2 * G


def region_slots(W: int, S: int) -> int:
    return (S + W + 2 + 31) // 32 * 32


def state_floats(G: int, D: int, W: int, S: int) -> int:
    return region_slots(W, S) * (ring_channels(G, D) + 2 * G * D) + D * D * G


def offsets(G: int, D: int, W: int, S: int):
    """(off_kp, off_vp, off_delta) in floats (bifrost.patch:1010-1013)."""
    LR, C = region_slots(W, S), ring_channels(G, D)
    off_kp = LR * C
    off_vp = off_kp + LR * G * D
    return off_kp, off_vp, off_vp + LR * G * D


def llama_slot(pos: int, W: int, S: int) -> int:
    """Region slot of position ``pos``'s ring row (bifrost.patch:848)."""
    WR = W + 1
    return S + ((pos % WR) + WR) % WR


def _views(row: torch.Tensor, G: int, D: int, W: int, S: int):
    LR, C = region_slots(W, S), ring_channels(G, D)
    off_kp, off_vp, off_dl = offsets(G, D, W, S)
    reg = row[:off_kp].view(LR, C)
    kp = row[off_kp:off_vp].view(G, LR, D)          # ggml [D, LR, G]
    vp = row[off_vp:off_dl].view(G, D, LR)          # ggml [LR, D, G]
    dl = row[off_dl:off_dl + D * D * G].view(G, D, D)   # [g, v, k]
    return reg, kp, vp, dl


def pack(cache: dict, next_pos, G: int, D: int, W: int, S: int) -> torch.Tensor:
    """Reference cache dict (B sequences) -> rows [B, state_floats] fp32.  ``next_pos`` [B]: each sequence's next
    position (the number of tokens it has seen).  ``ring_pos`` may be [W] (shared) or [B, W]."""
    rk, rv, rkm = cache["ring_k"], cache["ring_v"], cache["ring_km"]
    B = rk.shape[0]
    GD = G * D
    rows = torch.zeros(B, state_floats(G, D, W, S), dtype=torch.float32)
    rp = cache["ring_pos"]
    sk, sv, Sm = cache.get("sink_k"), cache.get("sink_v"), cache.get("S")
    for b in range(B):
        reg, kp, vp, dl = _views(rows[b], G, D, W, S)
        P = int(next_pos[b])
        rpb = rp[b] if rp.dim() == 2 else rp
        for p in range(max(0, P - W), P):            # the ring rows any later step reads
            j = p % W
            if int(rpb[j]) != p:
                continue
            l = llama_slot(p, W, S)
            k = rk[b, :, j].float()                  # [G, D]
            v = rv[b, :, j].float()
            reg[l, :GD] = k.reshape(-1)
            reg[l, GD:2 * GD] = v.reshape(-1)
            reg[l, 2 * GD:3 * GD] = rkm[b, j].float().reshape(-1)
            reg[l, 3 * GD:3 * GD + G] = cache["ring_g"][b, j].float()
            reg[l, 3 * GD + G:] = cache["ring_beta"][b, j].float()
            kp[:, l] = k
            vp[:, :, l] = v
        ns = 0 if sk is None else min(sk.shape[2], S, P)
        for l in range(ns):                          # sink slot l holds position l: k_rope | v only
            k = sk[b, :, l].float()
            v = sv[b, :, l].float()
            reg[l, :GD] = k.reshape(-1)
            reg[l, GD:2 * GD] = v.reshape(-1)
            kp[:, l] = k
            vp[:, :, l] = v
        if Sm is not None:
            dl.copy_(Sm[b].float().transpose(1, 2))
    return rows


def _bf16_rne(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> bf16 by round-to-nearest-even on the bit pattern (finite inputs)."""
    bits = x.float().contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    bits = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16
    hi = (bits << 16) & 0xFFFFFFFF
    hi = torch.where(hi >= 2 ** 31, hi - 2 ** 32, hi).to(torch.int32)
    return hi.view(torch.float32).to(torch.bfloat16)


def unpack(rows: torch.Tensor, next_pos, G: int, D: int, W: int, S: int, kv_dtype=torch.bfloat16,
           per_seq_pos: bool = True) -> dict:
    """Rows [B, state_floats] -> the reference cache dict for sequences at next positions ``next_pos`` [B].
    k_rope and v are rounded to ``kv_dtype`` (round-to-nearest-even for bf16).  ``ring_pos`` is [B, W] with
    ``per_seq_pos`` else [W] (then every sequence must be at the same position)."""
    B = rows.shape[0]
    GD = G * D
    cvt = _bf16_rne if kv_dtype == torch.bfloat16 else (lambda t: t.to(kv_dtype))
    out = dict(ring_k=torch.zeros(B, G, W, D, dtype=kv_dtype), ring_v=torch.zeros(B, G, W, D, dtype=kv_dtype),
               ring_km=torch.zeros(B, W, G, D), ring_g=torch.zeros(B, W, G), ring_beta=torch.zeros(B, W, G),
               ring_pos=torch.full((B, W), -1, dtype=torch.long), S=torch.zeros(B, G, D, D))
    P0 = [int(p) for p in next_pos]
    ns = min(S, min(P0)) if B else 0
    sink_k = torch.zeros(B, G, ns, D, dtype=kv_dtype)
    sink_v = torch.zeros(B, G, ns, D, dtype=kv_dtype)
    for b in range(B):
        reg, kp, vp, dl = _views(rows[b], G, D, W, S)
        P = P0[b]
        for p in range(max(0, P - W), P):
            j, l = p % W, llama_slot(p, W, S)
            out["ring_k"][b, :, j] = cvt(reg[l, :GD].view(G, D))
            out["ring_v"][b, :, j] = cvt(reg[l, GD:2 * GD].view(G, D))
            out["ring_km"][b, j] = reg[l, 2 * GD:3 * GD].view(G, D)
            out["ring_g"][b, j] = reg[l, 3 * GD:3 * GD + G]
            out["ring_beta"][b, j] = reg[l, 3 * GD + G:]
            out["ring_pos"][b, j] = p
        for l in range(ns):
            sink_k[b, :, l] = cvt(reg[l, :GD].view(G, D))
            sink_v[b, :, l] = cvt(reg[l, GD:2 * GD].view(G, D))
        out["S"][b] = dl.transpose(1, 2)
    if not per_seq_pos:
        out["ring_pos"] = out["ring_pos"][0].clone()
    out["sink_k"], out["sink_v"] = sink_k, sink_v
    return out


def llama_decode(row: torch.Tensor, p0: int, new: dict, qr, qm, mixx, mix_lse, mem_scale, G: int, D: int,
                 W: int, S: int, dtype=torch.float64):
    """One decode token at position ``p0`` of the port's graph on one sequence's row (modified in place).

    ``new``: this token's row parts k_rope [G,D], v [G,D], km [G,D], g [G], beta [G] (beta already masked by
    [p0 >= S]); qr [H,D] (RoPE'd query), qm [H,D] (the reference's memory query, unit(q fq) D^-1/2), mixx [H]
    (mix(x)), mix_lse, mem_scale [H].  Returns o [H,D] in ``dtype`` (before the output gate).
    """
    H = qr.shape[0]
    R = H // G
    GD = G * D
    LR = region_slots(W, S)
    reg, kp, vp, dl = _views(row, G, D, W, S)
    scratch = S + W + 1
    # the row leaving the window (read before any write, bifrost.patch:1042)
    wrow = reg[llama_slot(p0 - W, W, S)].clone()
    F = torch.cat([new[key].reshape(-1).float() for key in ("k_rope", "v", "km", "g", "beta")])
    s1 = p0 if p0 < S else scratch                   # sink slot of this token, or the scratch slot (:880)
    for l in (s1, llama_slot(p0, W, S)):             # region rows and both planes (:1043-1050)
        reg[l] = F
        kp[:, l] = F[:GD].view(G, D)
        vp[:, :, l] = F[GD:2 * GD].view(G, D)
    # mask over the LR region slots (:858-870)
    ok = torch.zeros(LR, dtype=torch.bool)
    for l in range(LR):
        if l < S:
            ok[l] = l <= p0
        elif l < scratch:
            r = l - S
            kpos = p0 - ((p0 - r) % (W + 1))
            ok[l] = kpos >= 0 and kpos >= S and p0 - kpos < W
    scale = 1.0 / math.sqrt(D)
    K = kp.to(dtype)                                  # [G, LR, D]
    V = vp.to(dtype)                                  # [G, D, LR]
    q = qr.to(dtype).view(G, R, D)
    kq = torch.einsum("grd,gld->grl", q, K) * scale
    kq = kq.masked_fill(~ok, float("-inf"))
    p = torch.softmax(kq, -1)
    # lse = E_p[s] + H(p), masked entries have p = 0 (:1097-1100)
    sfin = torch.where(ok, kq, torch.zeros_like(kq))
    lse = (p * sfin).sum(-1) - (p * torch.log(p.clamp(1e-30, 1.0))).sum(-1)
    o_win = torch.einsum("grl,gdl->grd", p, V).reshape(H, D)
    # memory: update the G states with the leaving row, read with the R query heads (:1115-1129)
    wk = wrow[2 * GD:3 * GD].view(G, D).to(dtype)
    wv = wrow[GD:2 * GD].view(G, D).to(dtype)
    wg = wrow[3 * GD:3 * GD + G].to(dtype)
    wb = wrow[3 * GD + G:].to(dtype)
    Sm = dl.to(dtype).transpose(1, 2) * wg.exp()[:, None, None]      # [g, k, v]
    delta = (wv - torch.einsum("gk,gkv->gv", wk, Sm)) * wb[:, None]
    Sm = Sm + wk[:, :, None] * delta[:, None, :]
    dl.copy_(Sm.transpose(1, 2).float())
    o_mem = torch.einsum("grk,gkv->grv", qm.to(dtype).view(G, R, D), Sm).reshape(H, D)
    # mix (:1145-1158)
    gamma = torch.sigmoid(mixx.to(dtype) + (lse.reshape(H) - math.log(W)) * mix_lse.to(dtype))
    gamma = gamma * (1.0 if p0 >= W else 0.0)
    om = o_mem * mem_scale.to(dtype)[:, None]
    return o_win + gamma[:, None] * (om - o_win)

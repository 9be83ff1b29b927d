"""CPU oracle for retrieval attention of the kept (not converted) full-attention layers.  TEST INFRASTRUCTURE ONLY.

Only ``tests/`` and ``bench.py``'s CPU legs may import this module; the product path
(``heimdall_b200.retrieval``) runs in CUDA with no CPU fallback.

It restates ``HybridAttention._teacher`` with its retrieval branch (reference project ``Heimdall``,
``heimdall/hibrit.py:275-324``):

* ``retrieval_mask`` -- ``_retrieval_mask`` (``hibrit.py:301-324``): per KV head, the query attends the sinks,
  the window from the block boundary at or before pos - W + 1, and the ``k`` candidate blocks with the largest
  upper bound of q.k over the block (max over the group's query heads of sum_d max(q_d kmax_d, q_d kmin_d),
  with the per-block key min / max: Quest-style block summaries).  Candidates are the full blocks that end before
  the window.
* ``teacher`` -- ``_teacher`` (``hibrit.py:275-290``): the cache-extended keys and values, then retrieval
  attention when it is on, applies (single-token decode, or prefill when ``prefill``) and there is history
  for ``k`` blocks, else causal attention over the whole cache; softmax in the compute dtype with scale D^-1/2.

Parity is pinned by the reference's own mask on seeded inputs (``tests/golden/golden_retrieval.pt`` made by
``tests/golden/make_golden.py``) and by the reference's properties: the mask equals a direct per-query
selection (``tests/test_hibrit.py:246-269``) and k covering every block gives full attention (``:231-243``).
"""
from __future__ import annotations

from typing import Optional

import torch


def block_bounds(qr, kr, block: int, sinks: int):
    """The upper bounds ub [B, G, t, nb] of q.k over each full block after the sinks (fp32, the reference's
    arithmetic): max over the group's query heads of sum_d (max(q_d, 0) kmax_d + min(q_d, 0) kmin_d)."""
    B, H, t, D = qr.shape
    G, n = kr.shape[1], kr.shape[2]
    R, S, L = H // G, sinks, block
    nb = (n - S) // L
    kb = kr[:, :, S:S + nb * L].float().reshape(B, G, nb, L, D)
    kmin, kmax = kb.amin(3), kb.amax(3)
    q = qr.float().reshape(B, G, R, t, D)
    ub = q.clamp(min=0) @ kmax[:, :, None].transpose(-1, -2) + q.clamp(max=0) @ kmin[:, :, None].transpose(-1, -2)
    return ub.amax(2)


def retrieval_mask(qr, kr, k: int, block: int, window: int, sinks: int):
    """Boolean mask [B, H, t, n] (True = attend) for the last t queries of qr [B,H,t,D] over kr [B,G,n,D]."""
    B, H, t, D = qr.shape
    G, n = kr.shape[1], kr.shape[2]
    R, S, W, L, K = H // G, sinks, window, block, k
    nb = (n - S) // L
    ub = block_bounds(qr, kr, L, S)                                       # [B, G, t, nb]
    qpos = torch.arange(n - t, n)
    nc = ((qpos - W + 1 - S).clamp(min=0) // L).clamp(max=nb)             # candidate blocks per query
    cand = torch.arange(nb)[None] < nc[:, None]                           # [t, nb]
    ub = ub.masked_fill(~cand, float("-inf"))
    top = ub.topk(min(K, nb), dim=-1).indices
    sel = torch.zeros(B, G, t, nb, dtype=torch.bool).scatter_(-1, top, True) & cand
    tok = torch.zeros(B, G, t, n, dtype=torch.bool)
    tok[..., S:S + nb * L] = sel.repeat_interleave(L, dim=-1)
    pos = torch.arange(n)
    base = (pos[None] < S) | ((pos[None] >= (S + nc * L)[:, None]) & (pos[None] <= qpos[:, None]))
    return (tok | base).repeat_interleave(R, dim=1)


def selected_blocks(qr, kr, k: int, block: int, window: int, sinks: int):
    """For a single query (t = 1): the candidate count nc and, per (b, g), the set of selected block indices."""
    mask = retrieval_mask(qr, kr, k, block, window, sinks)               # [B, H, 1, n]
    B, H, _, n = mask.shape
    G = kr.shape[1]
    R = H // G
    nb = (n - sinks) // block
    qpos = n - 1
    nc = max(0, min((qpos - window + 1 - sinks) // block, nb))
    out = []
    for b in range(B):
        row = []
        for g in range(G):
            m = mask[b, g * R, 0, sinks:sinks + nc * block].reshape(nc, block)[:, 0] if nc else torch.zeros(0)
            row.append(set(torch.nonzero(m).flatten().tolist()))
        out.append(row)
    return nc, out


def attend(qr, kr, vt, mask, dtype=torch.float64):
    """Softmax attention of qr [B,H,t,D] over kr/vt [B,G,n,D] with a boolean mask [B,H,t,n] -> o [B,t,H,D]."""
    B, H, t, D = qr.shape
    G = kr.shape[1]
    R = H // G
    k = kr.to(dtype).repeat_interleave(R, 1)
    v = vt.to(dtype).repeat_interleave(R, 1)
    s = (qr.to(dtype) @ k.transpose(-1, -2)) * D ** -0.5
    s = s.masked_fill(~mask, float("-inf"))
    return (s.softmax(-1) @ v).transpose(1, 2)


def teacher(qr, kr, v, cache: Optional[dict], retrieval: Optional[dict] = None, dtype=torch.float64):
    """``HybridAttention._teacher`` (hibrit.py:275-290): qr [B,H,t,D], kr [B,G,t,D], v [B,t,G,D] -> o [B,t,H,D];
    ``cache`` (or None) keeps "k", "v" [B,G,n,D]; ``retrieval`` is the dict of ``set_retrieval`` or None."""
    vt = v.transpose(1, 2)
    if cache is not None:
        if "k" in cache:
            kr, vt = torch.cat((cache["k"], kr), 2), torch.cat((cache["v"], vt), 2)
        cache["k"], cache["v"] = kr, vt
    t, n = qr.shape[2], kr.shape[2]
    ret = retrieval
    if ret is not None and (t == 1 or ret.get("prefill")) and n - ret["sinks"] - ret["window"] >= ret["k"] * ret["block"]:
        mask = retrieval_mask(qr, kr, ret["k"], ret["block"], ret["window"], ret["sinks"])
    else:
        B, H = qr.shape[:2]
        mask = (torch.arange(n)[None] <= torch.arange(n - t, n)[:, None]).expand(B, H, t, n)
    return attend(qr, kr, vt, mask, dtype)

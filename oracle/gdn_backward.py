"""CPU oracle for the backward of the GQA gated delta rule.  TEST INFRASTRUCTURE ONLY.

Only ``tests/`` and ``bench.py``'s CPU legs import this module; the CUDA path in ``heimdall_b200`` never calls
into it.

The reference differentiates ``delta_rule_gqa`` (``heimdall/motor.py:70-102``) with torch autograd when
``seq_loss`` (``heimdall/motor.py:149-193``) trains a converted layer; the loss and gradient pins of that path are
``tests/test_motor.py:42-65``.  The checker for the GPU backward is therefore torch autograd through this repo's
restatement of the forward (``oracle.bifrost_oracle.gdn_gqa``, fp64), which ``autograd_grads`` runs.

``recurrent_grads`` restates the same gradients as the explicit token-by-token reverse recurrence that
``csrc/gdn_backward.cu`` computes, so the CPU tests can check that derivation against autograd:

    forward:  S~ = a S_{t-1} (a = e^g),  e = v - S~^T k,  S_t = S~ + beta k e^T,  o_r = S_t^T q_r
    backward: dS += sum_r q_r do_r^T;  dq_r = S_t do_r;  kds = dS^T k;  de = beta kds;  dv = de;
              dbeta = e . kds;  dk = beta dS e - S~ de;  dS~ = dS - k de^T;  dg = <dS~, S~>;  dS_{t-1} = a dS~
"""
from __future__ import annotations

import torch

from .bifrost_oracle import gdn_gqa


def autograd_grads(q, k, v, g, beta, s0, do, dsT, chunk: int = 64, dtype=torch.float64):
    """Gradients of sum(o * do) + sum(S_T * dsT) through the fp64 chunked forward (the reference's autograd).

    q [B,T,G,R,D]; k, v [B,T,G,D]; g, beta [B,T,G]; s0 [B,G,D,D] or None; do like the output; dsT like the state or
    None.  Returns (dq, dk, dv, dg, dbeta, ds0)."""
    leaves = [t.detach().to(dtype).requires_grad_(True) for t in (q, k, v, g, beta)]
    st = None if s0 is None else s0.detach().to(dtype).requires_grad_(True)
    o, S = gdn_gqa(*leaves, chunk=chunk, state=st, dtype=dtype)
    loss = (o * do.to(dtype)).sum()
    if dsT is not None:
        loss = loss + (S * dsT.to(dtype)).sum()
    want = leaves + ([st] if st is not None else [])
    grads = torch.autograd.grad(loss, want)
    ds0 = grads[5] if st is not None else None
    return (*grads[:5], ds0)


def recurrent_grads(q, k, v, g, beta, s0, do, dsT, dtype=torch.float64):
    """The explicit reverse recurrence (see the module docstring); same arguments and results as
    ``autograd_grads``, ds0 always returned."""
    q, k, v, g, beta, do = (t.to(dtype) for t in (q, k, v, g, beta, do))
    B, T, G, R, D = q.shape
    S = torch.zeros(B, G, D, D, dtype=dtype) if s0 is None else s0.to(dtype).clone()
    states, errs = [S], []
    for t in range(T):                                       # forward, keeping every state
        a = g[:, t].exp()[..., None, None]
        St = a * S
        e = v[:, t] - torch.einsum("bgij,bgi->bgj", St, k[:, t])
        S = St + beta[:, t][..., None, None] * k[:, t][..., :, None] * e[..., None, :]
        states.append(S)
        errs.append(e)
    dS = torch.zeros(B, G, D, D, dtype=dtype) if dsT is None else dsT.to(dtype).clone()
    dq, dk, dv = torch.zeros_like(q), torch.zeros_like(k), torch.zeros_like(v)
    dg, db = torch.zeros_like(g), torch.zeros_like(beta)
    for t in range(T - 1, -1, -1):
        St, Sp, e = states[t + 1], states[t], errs[t]
        kt, bt, a = k[:, t], beta[:, t], g[:, t].exp()
        dS = dS + torch.einsum("bgri,bgrj->bgij", q[:, t], do[:, t])
        dq[:, t] = torch.einsum("bgij,bgrj->bgri", St, do[:, t])
        kds = torch.einsum("bgij,bgi->bgj", dS, kt)
        de = bt[..., None] * kds
        dv[:, t] = de
        db[:, t] = (e * kds).sum(-1)
        Stl = a[..., None, None] * Sp
        dk[:, t] = bt[..., None] * torch.einsum("bgij,bgj->bgi", dS, e) - torch.einsum("bgij,bgj->bgi", Stl, de)
        dSt = dS - kt[..., :, None] * de[..., None, :]
        dg[:, t] = (dSt * Stl).sum((-1, -2))
        dS = a[..., None, None] * dSt
    return dq, dk, dv, dg, db, dS

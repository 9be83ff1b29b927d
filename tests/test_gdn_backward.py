"""The backward of the GQA gated delta rule on the CPU: the explicit reverse recurrence that
``csrc/gdn_backward.cu`` computes (``oracle/gdn_backward.py``) against torch autograd through the fp64 forward
oracle, which is how the reference differentiates ``delta_rule_gqa`` (heimdall/motor.py:70-102) in ``seq_loss``
(motor.py:149-193)."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle import gdn_backward as ogb
from oracle.bifrost_oracle import rel_l2


def _case(B, T, G, R, D, seed, with_state=True):
    gen = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=gen, dtype=torch.float64)
    q = F.normalize(r(B, T, G, R, D), dim=-1) * D ** -0.5
    k = F.normalize(r(B, T, G, D), dim=-1)
    v = r(B, T, G, D)
    g = -torch.rand(B, T, G, generator=gen, dtype=torch.float64) * 0.3
    beta = torch.rand(B, T, G, generator=gen, dtype=torch.float64)
    s0 = r(B, G, D, D) * 0.1 if with_state else None
    do = r(B, T, G, R, D)
    dsT = r(B, G, D, D) * 0.1 if with_state else None
    return q, k, v, g, beta, s0, do, dsT


@pytest.mark.parametrize("B,T,G,R,D,state", [(2, 37, 2, 3, 8, True), (1, 70, 1, 2, 16, False), (1, 5, 3, 1, 4, True)])
def test_recurrent_backward_equals_autograd(B, T, G, R, D, state):
    args = _case(B, T, G, R, D, seed=T + D, with_state=state)
    got = ogb.recurrent_grads(*args)
    want = ogb.autograd_grads(*args, chunk=16)
    for name, x, y in zip(("dq", "dk", "dv", "dg", "dbeta", "ds0"), got, want):
        if y is None:
            continue
        assert rel_l2(x, y) < 1e-10, name


def test_chunk_length_does_not_change_gradients():
    """The chunked forward's gradients are those of the recurrence whatever the chunk (the GPU scan uses 128)."""
    args = _case(1, 50, 2, 2, 8, seed=5)
    a = ogb.autograd_grads(*args, chunk=8)
    b = ogb.autograd_grads(*args, chunk=64)
    for x, y in zip(a, b):
        assert rel_l2(x, y) < 1e-10

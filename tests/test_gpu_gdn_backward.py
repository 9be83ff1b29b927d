"""GPU parity of the delta-rule backward (``bf_gdn_bwd`` through ``functional.delta_rule_gqa_backward`` and the
autograd path of ``functional.delta_rule_gqa``) against torch autograd through the fp64 forward oracle: the
gradients the reference's ``seq_loss`` (heimdall/motor.py:149-193) takes through ``delta_rule_gqa``
(motor.py:70-102).

Tolerance: rel-L2 <= 1e-4 per gradient (fp32 recurrence against fp64).  The autograd path's forward runs the
tensor-core scan (fp16 operands), so its loss carries the forward's 1e-3-level error; its gradients come from
the fp32 backward and are held to the same 1e-4.
"""
import pytest
import torch
import torch.nn.functional as F

from oracle import gdn_backward as ogb
from oracle.bifrost_oracle import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-4
NAMES = ("dq", "dk", "dv", "dg", "dbeta", "ds0")


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


def _case(B, T, G, R, seed, with_state=True, D=256):
    gen = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=gen)
    q = F.normalize(r(B, T, G, R, D), dim=-1) * D ** -0.5
    k = F.normalize(r(B, T, G, D), dim=-1)
    v = r(B, T, G, D)
    g = -torch.rand(B, T, G, generator=gen) * 0.5
    g[..., 0] = 0.0                                   # an archival head: never forgets
    beta = torch.rand(B, T, G, generator=gen)
    s0 = r(B, G, D, D) * 0.05 if with_state else None
    do = r(B, T, G, R, D)
    dsT = r(B, G, D, D) * 0.05 if with_state else None
    return q, k, v, g, beta, s0, do, dsT


@pytest.mark.parametrize("B,T,G,R,state", [(2, 150, 2, 3, True), (1, 64, 1, 6, False), (1, 1, 2, 2, True),
                                           (1, 300, 4, 6, True)])
def test_backward_matches_autograd_oracle(B, T, G, R, state):
    dev = _dev()
    from heimdall_b200.functional import delta_rule_gqa_backward
    args = _case(B, T, G, R, seed=T * 7 + G, with_state=state)
    want = ogb.autograd_grads(*args)
    cu = [None if t is None else t.to(dev) for t in args]
    got = delta_rule_gqa_backward(*cu)
    torch.cuda.synchronize()
    for name, x, y in zip(NAMES, got, want):
        if y is None:
            continue
        assert rel_l2(x.cpu().double(), y) < TOL, name


def test_autograd_path_two_segments_with_state_carry():
    """seq_loss's shape of use: two segments, the second starting from the first's final state, the loss a
    weighted square of both outputs; gradients w.r.t. q, k, g, beta of both segments and the initial state."""
    dev = _dev()
    from heimdall_b200.functional import delta_rule_gqa
    B, G, R, D = 1, 2, 3, 256
    a1 = _case(B, 90, G, R, seed=1)
    a2 = _case(B, 70, G, R, seed=2)
    w1, w2 = torch.randn(B, 90, G, R, D), torch.randn(B, 70, G, R, D)

    def run(fn, dev_, dtype):
        leaves = [t.to(dev_, dtype).requires_grad_(True) for t in (*a1[:5], *a2[:5], a1[5])]
        (q1, k1, v1, g1, b1, q2, k2, v2, g2, b2, s0) = leaves
        o1, s1 = fn(q1, k1, v1, g1, b1, s0)
        o2, _ = fn(q2, k2, v2, g2, b2, s1)
        loss = ((o1 * w1.to(dev_, dtype)) ** 2).sum() + ((o2 * w2.to(dev_, dtype)) ** 2).sum()
        grads = torch.autograd.grad(loss, leaves)
        return loss.detach(), grads

    from oracle.bifrost_oracle import gdn_gqa
    ref_loss, ref = run(lambda q, k, v, g, b, s: gdn_gqa(q, k, v, g, b, 64, s, torch.float64), "cpu", torch.float64)
    loss, got = run(lambda q, k, v, g, b, s: delta_rule_gqa(q, k, v, g, b, 64, s), dev, torch.float32)
    torch.cuda.synchronize()
    assert abs(loss.item() - ref_loss.item()) < 5e-3 * abs(ref_loss.item())
    # the loss gradient do = 2 w^2 o uses the forward's o (tensor-core scan, ~1e-3): compare at that level
    for i, (x, y) in enumerate(zip(got, ref)):
        assert rel_l2(x.cpu().double(), y) < 5e-3, i


def test_backward_rejects_bad_shapes():
    dev = _dev()
    from heimdall_b200 import _lib
    from heimdall_b200.functional import delta_rule_gqa_backward
    z = lambda *s: torch.zeros(*s, device=dev)
    with pytest.raises(NotImplementedError):
        delta_rule_gqa_backward(z(1, 4, 1, 1, 64), z(1, 4, 1, 64), z(1, 4, 1, 64), z(1, 4, 1), z(1, 4, 1), None, None,
                                None)
    assert _lib.size("bf_gdn_bwd_workspace", 1, 4, 1, 9, 256) == 0     # R > 8

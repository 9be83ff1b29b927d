"""Retrieval attention of the kept full-attention layers on the CPU: the oracle against the reference's own mask
and attention (golden fixtures made by running ``HybridAttention._retrieval_mask``), and the reference's
properties of the path (``tests/test_hibrit.py:231-269``)."""
from __future__ import annotations

from pathlib import Path

import pytest
import torch

from oracle import retrieval as orr

from conftest import reference_project

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("name", ["small", "decode_d256", "prefill_d64"])
def test_oracle_mask_and_output_match_reference(golden_retrieval, name):
    c = golden_retrieval[name]
    ret = c["ret"]
    qr, kr, vt = c["qr"].float(), c["kr"].float(), c["vt"].float()
    mask = orr.retrieval_mask(qr, kr, ret["k"], ret["block"], ret["window"], ret["sinks"])
    assert torch.equal(mask, c["mask"])
    o = orr.attend(qr, kr, vt, mask)
    torch.testing.assert_close(o, c["o"].double(), rtol=1e-5, atol=1e-5)


def test_mask_is_direct_per_query_selection():
    """The mask equals a direct selection per query and KV head: sinks, the window from the block boundary, and
    the top-k candidate blocks by upper bound (the reference's own check, test_hibrit.py:246-269)."""
    torch.manual_seed(0)
    B, H, G, D, n, t = 1, 4, 2, 8, 50, 3
    qr, kr = torch.randn(B, H, t, D), torch.randn(B, G, n, D)
    S, W, L, R, K = 2, 6, 4, H // G, 2
    mask = orr.retrieval_mask(qr, kr, K, L, W, S)
    for g in range(G):
        for i in range(t):
            p = n - t + i
            blocks = [b for b in range((n - S) // L) if S + (b + 1) * L <= p - W + 1]
            ub = {b: max(sum(max(qr[0, h, i, d] * kr[0, g, S + b * L:S + (b + 1) * L, d].min(),
                                 qr[0, h, i, d] * kr[0, g, S + b * L:S + (b + 1) * L, d].max()) for d in range(D))
                         for h in range(g * R, (g + 1) * R)) for b in blocks}
            top = sorted(blocks, key=lambda b: -ub[b])[:K]
            want = torch.zeros(n, dtype=torch.bool)
            want[:S] = True
            want[S + len(blocks) * L:p + 1] = True
            for b in top:
                want[S + b * L:S + (b + 1) * L] = True
            for h in range(g * R, (g + 1) * R):
                assert torch.equal(mask[0, h, i], want), (g, i)


def test_every_block_selected_equals_full_attention():
    """k covering every block gives exactly causal attention over the whole cache (test_hibrit.py:231-243)."""
    torch.manual_seed(1)
    B, H, G, D, n = 1, 4, 2, 16, 90
    qr, kr, v = torch.randn(B, H, 1, D), torch.randn(B, G, n, D), torch.randn(B, 1, G, D)
    cache = {"k": kr[:, :, :-1], "v": v.new_zeros(B, G, n - 1, D).normal_()}
    full = orr.teacher(qr, kr[:, :, -1:], v, dict(cache), None)
    ret = dict(k=100, block=4, window=8, sinks=2)
    got = orr.teacher(qr, kr[:, :, -1:], v, dict(cache), ret)
    torch.testing.assert_close(got, full, rtol=1e-12, atol=1e-12)


def test_reference_mask_live():
    """With the reference present, its _retrieval_mask runs here once more on fresh inputs."""
    proj = reference_project()
    if proj is None:
        pytest.skip("HEIMDALL_REFERENCE not set")
    import sys
    sys.path.insert(0, str(proj))
    import heimdall.hibrit as hb
    torch.manual_seed(3)
    qr, kr = torch.randn(2, 12, 1, 32), torch.randn(2, 3, 400, 32)
    ret = dict(k=5, block=8, window=64, sinks=4)
    assert torch.equal(orr.retrieval_mask(qr, kr, 5, 8, 64, 4), hb.HybridAttention._retrieval_mask(None, qr, kr, ret))

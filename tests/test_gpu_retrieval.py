"""GPU parity of the kept layers' attention (``heimdall_b200.retrieval.teacher``: HybridAttention._teacher with its
retrieval branch) against the reference's own outputs (golden fixture) and the CPU oracle (``oracle/retrieval.py``).

Tolerances: outputs rel-L2 <= 2e-3 (bf16 cache, fp32 softmax).  The block selection is an arg-top-k of fp32
bounds whose summation order differs from the reference's matmul; the production-geometry tests check that the
k-th and (k+1)-th bounds of every (sequence, KV head) are apart by more than that rounding before comparing.
"""
import pytest
import torch

from oracle import retrieval as orr
from oracle.bifrost_oracle import rel_l2

pytestmark = pytest.mark.gpu
O_TOL = 2e-3


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


def _margin_ok(qr, kr, ret):
    """The k-th and (k+1)-th candidate bounds differ by more than fp32 summation-order noise everywhere."""
    S, W, L, K = ret["sinks"], ret["window"], ret["block"], ret["k"]
    n = kr.shape[2]
    ub = orr.block_bounds(qr.float(), kr.float(), L, S).double()          # [B, G, 1, nb]
    nc = max(0, min((n - W - S) // L, (n - S) // L))
    top = ub[..., :nc].sort(-1, descending=True).values
    if nc <= K:
        return True
    gap = (top[..., K - 1] - top[..., K]).abs()
    return bool((gap > 3e-5 * top[..., 0].abs().clamp_min(1.0)).all())


def test_decode_matches_reference_golden(golden_retrieval):
    """The reference's _teacher decode with retrieval (24 query / 4 KV heads, D = 256), from its own cache."""
    dev = _dev()
    from heimdall_b200.retrieval import teacher
    c = golden_retrieval["decode_d256"]
    ret = c["ret"]
    qr, kr, vt = c["qr"], c["kr"], c["vt"]
    cache = {"k": kr[:, :, :-1].to(dev), "v": vt[:, :, :-1].to(dev)}
    o = teacher(qr.to(dev), kr[:, :, -1:].to(dev), vt[:, :, -1:].transpose(1, 2).to(dev), cache, ret)
    torch.cuda.synchronize()
    assert rel_l2(o.float().cpu(), c["o"]) < O_TOL
    assert torch.equal(cache["k"].cpu(), kr)


@pytest.mark.parametrize("B,n", [(2, 40000), (3, 9000)])
def test_decode_production_geometry(B, n):
    """k = 16 blocks of 64, window 2048, 4 sinks, 24 query / 4 KV heads: one decode token against the oracle."""
    dev = _dev()
    from heimdall_b200.retrieval import teacher
    H, G, D = 24, 4, 256
    ret = dict(k=16, block=64, window=2048, sinks=4)
    bf = torch.bfloat16
    for seed in range(n + B, n + B + 20):      # inputs without a near-tie at the k-th block of any (b, g)
        gen = torch.Generator().manual_seed(seed)
        qr = torch.randn(B, H, 1, D, generator=gen).to(bf)
        kr = torch.randn(B, G, n, D, generator=gen).to(bf)
        vt = torch.randn(B, G, n, D, generator=gen).to(bf)
        if _margin_ok(qr, kr, ret):
            break
    else:
        pytest.fail("no seed without a near-tie")
    o_ref = orr.teacher(qr.float(), kr[:, :, -1:].float(), vt[:, :, -1:].transpose(1, 2).float(),
                        {"k": kr[:, :, :-1].float(), "v": vt[:, :, :-1].float()}, ret)
    cache = {"k": kr[:, :, :-1].to(dev), "v": vt[:, :, :-1].to(dev)}
    o = teacher(qr.to(dev), kr[:, :, -1:].to(dev), vt[:, :, -1:].transpose(1, 2).to(dev), cache, ret)
    torch.cuda.synchronize()
    assert rel_l2(o.float().cpu(), o_ref) < O_TOL


def test_prefill_then_decode_steps_with_growing_cache():
    """A causal prefill of 1500 tokens (window kernel over the whole cache), then decode steps across block
    boundaries: the summaries follow the cache as blocks fill and the capacity grows (1024 -> 2048)."""
    dev = _dev()
    from heimdall_b200.retrieval import teacher
    B, H, G, D = 1, 8, 2, 256
    ret = dict(k=3, block=32, window=256, sinks=4)
    T0, steps = 1500, 40
    gen = torch.Generator().manual_seed(7)
    bf = torch.bfloat16
    qr = torch.randn(B, H, T0 + steps, D, generator=gen).to(bf)
    kr = torch.randn(B, G, T0 + steps, D, generator=gen).to(bf)
    v = torch.randn(B, T0 + steps, G, D, generator=gen).to(bf)
    cache, cache_r = {}, {}
    o = teacher(qr[:, :, :T0].to(dev), kr[:, :, :T0].to(dev), v[:, :T0].to(dev), cache, ret)
    o_ref = orr.teacher(qr[:, :, :T0].float(), kr[:, :, :T0].float(), v[:, :T0].float(), cache_r, ret)
    torch.cuda.synchronize()
    assert rel_l2(o.float().cpu(), o_ref) < O_TOL
    checked = 0
    for i in range(T0, T0 + steps):
        qs, ks = qr[:, :, i:i + 1], kr[:, :, i:i + 1]
        o = teacher(qs.to(dev), ks.to(dev), v[:, i:i + 1].to(dev), cache, ret)
        o_ref = orr.teacher(qs.float(), ks.float(), v[:, i:i + 1].float(), cache_r, ret)
        torch.cuda.synchronize()
        if _margin_ok(qs, kr[:, :, :i + 1], ret):   # a near-tie at the k-th block may select either
            assert rel_l2(o.float().cpu(), o_ref) < O_TOL, i
            checked += 1
    assert checked >= steps // 2
    assert cache["_cap"] == 2048 and cache["_ret_nb"] == (T0 + steps - 4) // 32


def test_prefill_with_retrieval_raises():
    """Retrieval in prefill (a selection per query) is not built: it raises instead of computing something else."""
    dev = _dev()
    from heimdall_b200.retrieval import teacher
    z = lambda *s: torch.zeros(*s, dtype=torch.bfloat16, device=dev)
    ret = dict(k=2, block=16, window=64, sinks=4, prefill=True)
    cache = {"k": z(1, 1, 595, 256), "v": z(1, 1, 595, 256)}
    with pytest.raises(NotImplementedError):
        teacher(z(1, 2, 5, 256), z(1, 1, 5, 256), z(1, 5, 1, 256), cache, ret)

"""The llama.cpp state-row interchange on the CPU: the oracle's row format against the reference's layer
semantics, the GGUF tensors against the reference's own converter, and the C ABI's size query.

The state row has no golden vectors in the reference (its port runs only inside llama.cpp), so the format is
pinned by behaviour: a row packed from a cache that the reference-pinned oracle ``student`` built, advanced by
one token of the port's decode graph (``oracle.llama_state.llama_decode``), must give the output of the
reference's own decode of that cache and unpack to the cache the reference leaves behind.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tests" / "golden"))
from oracle import bifrost_oracle as orc  # noqa: E402
from oracle import llama_state as ls  # noqa: E402
from params import layer_params  # noqa: E402

from conftest import reference_project  # noqa: E402

H, G, D, d, W, S = 4, 2, 16, 32, 8, 2


def _tokens(B, t, gen, dtype=torch.float32):
    n = lambda *s: torch.randn(*s, generator=gen, dtype=torch.float64).to(dtype)
    return dict(x=n(B, t, d), q=n(B, t, H, D), k=n(B, t, G, D), v=n(B, t, G, D), qr=n(B, H, t, D), kr=n(B, G, t, D))


def _clone(c):
    return {k: (v.clone() if torch.is_tensor(v) else v) for k, v in c.items()}


def test_geometry_matches_port_formula():
    assert ls.ring_channels(4, 256) == 3080
    assert ls.region_slots(2048, 4) == 2080
    assert ls.state_floats(4, 256, 2048, 4) == 2080 * (3080 + 2048) + 256 * 256 * 4
    off_kp, off_vp, off_dl = ls.offsets(4, 256, 2048, 4)
    assert (off_kp, off_vp - off_kp, off_dl - off_vp) == (2080 * 3080, 2080 * 1024, 2080 * 1024)
    assert [ls.llama_slot(p, 8, 2) for p in (-1, 0, 7, 8, 9, 18)] == [10, 2, 9, 10, 2, 2]


def test_capi_size_query_matches_oracle():
    from heimdall_b200 import _lib
    for geo in ((4, 256, 2048, 4), (2, 16, 8, 2), (1, 32, 100, 0)):
        assert _lib.size("bf_llama_state_floats", *geo) == ls.state_floats(*geo)
    assert _lib.size("bf_llama_state_floats", 0, 256, 2048, 4) == 0


def test_bf16_rounding_is_nearest_even():
    x = torch.randn(100000, dtype=torch.float32) * 10
    x = torch.cat((x, torch.tensor([1.00390625, 1.01171875, -2.0078125, 0.0, -0.0])))   # ties both ways
    assert torch.equal(ls._bf16_rne(x).view(torch.int16), x.to(torch.bfloat16).view(torch.int16))


@pytest.mark.parametrize("T0", [1, 2, 5, 7, 8, 9, 13, 30])
def test_packed_row_continues_like_reference(T0):
    """pack(cache) -> one port decode token == the reference's decode of the cache, and the row after it
    unpacks to the reference's cache after it."""
    p = layer_params(H, G, D, d, W, S, archival=1, seed=5)
    gen = torch.Generator().manual_seed(T0)
    B = 2
    pre = _tokens(B, T0, gen)
    cache = {}
    orc.student(p, pre["x"], pre["q"], pre["k"], pre["v"], pre["qr"], pre["kr"], 0, cache, dtype=torch.float64)
    rows = ls.pack(cache, [T0] * B, G, D, W, S)
    assert rows.shape == (B, ls.state_floats(G, D, W, S))
    nxt = _tokens(B, 1, gen)
    ref_cache = _clone(cache)
    o_ref = orc.student(p, nxt["x"], nxt["q"], nxt["k"], nxt["v"], nxt["qr"], nxt["kr"], T0, ref_cache,
                        dtype=torch.float64)
    pos = torch.tensor([T0])
    qm, km, g, beta = orc.mem_inputs(p, nxt["x"], nxt["q"], nxt["k"], pos, dtype=torch.float64)
    mixx = nxt["x"].double() @ p.mix_w.double().t() + p.mix_b.double()
    for b in range(B):
        new = dict(k_rope=nxt["kr"][b, :, 0], v=nxt["v"][b, 0], km=km[b, 0], g=g[b, 0], beta=beta[b, 0])
        o = ls.llama_decode(rows[b], T0, new, nxt["qr"][b, :, 0], qm[b, 0], mixx[b, 0], p.mix_lse, p.mem_scale,
                            G, D, W, S)
        torch.testing.assert_close(o, o_ref[b, 0].double(), rtol=1e-5, atol=1e-5)
    back = ls.unpack(rows, [T0 + 1] * B, G, D, W, S, kv_dtype=torch.float32, per_seq_pos=False)
    valid = ref_cache["ring_pos"] >= 0
    assert torch.equal(back["ring_pos"], ref_cache["ring_pos"])
    for key in ("ring_k", "ring_v"):
        torch.testing.assert_close(back[key][:, :, valid], ref_cache[key][:, :, valid].float(), rtol=0, atol=0)
    for key in ("ring_km", "ring_g", "ring_beta"):
        torch.testing.assert_close(back[key][:, valid], ref_cache[key][:, valid].float(), rtol=1e-6, atol=1e-7)
    ns = min(S, T0 + 1)
    torch.testing.assert_close(back["sink_k"], ref_cache["sink_k"][:, :, :ns].float(), rtol=0, atol=0)
    S_ref = ref_cache.get("S", torch.zeros(B, G, D, D))
    torch.testing.assert_close(back["S"], S_ref.float(), rtol=1e-5, atol=1e-6)


def test_round_trip_bf16_cache_is_exact_and_rows_zero_elsewhere():
    p = layer_params(H, G, D, d, W, S, archival=1, seed=6)
    gen = torch.Generator().manual_seed(1)
    B, T0 = 3, 21
    pre = _tokens(B, T0, gen, torch.bfloat16)
    cache = {}
    orc.student(p, pre["x"], pre["q"], pre["k"], pre["v"], pre["qr"], pre["kr"], 0, cache)
    rows = ls.pack(cache, [T0] * B, G, D, W, S)
    back = ls.unpack(rows, [T0] * B, G, D, W, S, per_seq_pos=False)
    for key in ("ring_k", "ring_v", "ring_km", "ring_g", "ring_beta", "ring_pos", "sink_k", "sink_v", "S"):
        assert back[key].dtype == cache[key].dtype, key
        assert torch.equal(back[key], cache[key]), key
    # the stale (W+1)-th ring slot, scratch and padding are zero in every plane
    reg, kp, vp, _ = ls._views(rows[0], G, D, W, S)
    dead = [ls.llama_slot(T0 - W - 1, W, S)] + list(range(S + W + 1, ls.region_slots(W, S)))
    assert not reg[dead].any() and not kp[:, dead].any() and not vp[:, :, dead].any()
    # planes mirror the region
    live = [l for l in range(ls.region_slots(W, S)) if l not in dead]
    GD = G * D
    assert torch.equal(kp[:, live].permute(1, 0, 2).reshape(len(live), GD), reg[live, :GD])
    assert torch.equal(vp[:, :, live].permute(2, 0, 1).reshape(len(live), GD), reg[live, GD:2 * GD])


def test_row_of_short_sequence_keeps_only_seen_positions():
    """Before the ring fills, slots of positions not yet seen stay zero; unpack marks them empty."""
    p = layer_params(H, G, D, d, W, S, archival=0, seed=7)
    gen = torch.Generator().manual_seed(2)
    pre = _tokens(1, 3, gen, torch.bfloat16)
    cache = {}
    orc.student(p, pre["x"], pre["q"], pre["k"], pre["v"], pre["qr"], pre["kr"], 0, cache)
    rows = ls.pack(cache, [3], G, D, W, S)
    reg = ls._views(rows[0], G, D, W, S)[0]
    seen = {ls.llama_slot(t, W, S) for t in range(3)} | {0, 1}
    for l in range(ls.region_slots(W, S)):
        assert bool(reg[l].any()) == (l in seen), l
    back = ls.unpack(rows, [3], G, D, W, S)
    assert back["ring_pos"][0].tolist() == [0, 1, 2] + [-1] * (W - 3)


# ------------------------------------------------------------------------------------------ GGUF tensors
@pytest.fixture(scope="module")
def golden_gguf():
    return torch.load(ROOT / "tests" / "golden" / "golden_gguf.pt", weights_only=False)


def test_gguf_tensors_match_reference_converter(golden_gguf):
    from heimdall_b200.interchange import GGUF_TENSORS, gguf_metadata, gguf_tensors
    assert golden_gguf["window"] == 16 and golden_gguf["sinks"] == 4
    for idx, params in golden_gguf["layers"].items():
        ours = gguf_tensors(params)
        ref = golden_gguf["tensors"][idx]
        assert set(ours) == set(ref) == set(GGUF_TENSORS)
        for name in GGUF_TENSORS:
            assert ours[name].dtype == ref[name].numpy().dtype, name
            assert ours[name].shape == tuple(ref[name].shape), name
            assert (ours[name] == ref[name].numpy()).all(), name
    meta = gguf_metadata(16, 4, golden_gguf["layers"].keys(), 8)
    assert meta == {"qwen35.bifrost.window": 16, "qwen35.bifrost.sinks": 4,
                    "qwen35.bifrost.layers": [0, 0, 0, 1, 0, 0, 0, 1]}


def test_params_from_gguf_inverts_the_export(golden_gguf):
    from heimdall_b200.interchange import gguf_tensors, params_from_gguf
    for idx, params in golden_gguf["layers"].items():
        back = params_from_gguf({k: v.numpy() for k, v in golden_gguf["tensors"][idx].items()})
        for name in ("fq", "fk", "ab_w", "ab_b", "mix_w", "mix_b", "mix_lse", "mem_scale", "dt_bias", "decay_mask"):
            assert torch.equal(back[name], params[name].float()), name
        live = params["decay_mask"] != 0
        torch.testing.assert_close(back["A_log"][live], params["A_log"][live], rtol=1e-6, atol=1e-6)
        again = gguf_tensors(back)
        for name, arr in again.items():
            torch.testing.assert_close(torch.from_numpy(arr), golden_gguf["tensors"][idx][name], rtol=1e-6, atol=0)


def test_gguf_tensors_live_reference():
    """With the reference present, its converter runs here on the golden parameters once more."""
    proj = reference_project()
    if proj is None or not (proj / "llamacpp" / "bifrost_gguf.py").is_file():
        pytest.skip("HEIMDALL_REFERENCE not set")
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    import make_golden
    from heimdall_b200.interchange import gguf_tensors
    case = make_golden.gguf_case(proj)
    for idx, params in case["layers"].items():
        ours = gguf_tensors(params)
        for name, t in case["tensors"][idx].items():
            assert (ours[name] == t.numpy()).all(), name

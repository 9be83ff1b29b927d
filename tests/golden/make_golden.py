"""Generate the golden fixtures in this folder by running the REFERENCE implementation.

Run where the reference project is available, naming its directory (the one that holds ``Heimdall/``, or
``Heimdall/`` itself) with ``--ref`` or the environment variable HEIMDALL_REFERENCE::

    HEIMDALL_REFERENCE=<reference checkout> python tests/golden/make_golden.py

It imports Heimdall's own ``heimdall.kernels``, ``heimdall.motor`` and ``heimdall.hibrit`` and runs
them, unmodified, on seeded inputs.  Inputs and outputs are saved to ``golden_*.pt``.  Inputs that
feed the bf16 CUDA path are rounded to bf16 first, so the same values can be handed to the kernels.
The large D=256 parameter tensors are not stored: they are regenerated from a seed by
``tests/golden/params.py`` and the fixture keeps their checksums to detect any drift.
"""
from __future__ import annotations

import argparse
import math
import os
import sys
from pathlib import Path

import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from params import make_module_params, make_module_proj, module_config, param_tensors  # noqa: E402


def bf(x):
    """Round to bf16 values, keep fp32 storage."""
    return x.to(torch.bfloat16).float()


def gdn_cases(hk, hm):
    out = {}
    # chunked == recurrent pin, shapes of tests/test_heimdall.py:36-48
    torch.manual_seed(0)
    b, t, h, d = 2, 45, 2, 16
    q = F.normalize(torch.randn(b, t, h, d), dim=-1) * d ** -0.5
    k = F.normalize(torch.randn(b, t, h, d), dim=-1)
    v, g, beta = torch.randn(b, t, h, d), -torch.rand(b, t, h) * 0.3, torch.rand(b, t, h)
    s0 = torch.randn(b, h, d, d) * 0.1
    o, s = hk.delta_rule_reference(q, k, v, g, beta, 16, s0)
    st, outs = s0, []
    for i in range(t):
        oi, st = hk.delta_rule_step(q[:, i], k[:, i], v[:, i], g[:, i], beta[:, i], st)
        outs.append(oi)
    out["gdn_small"] = dict(q=q, k=k, v=v, g=g, beta=beta, s0=s0, chunk=16, o=o, S=s,
                            o_rec=torch.stack(outs, 1), S_rec=st)
    # the prepare() self-test case (kernels.py:168-178): b=2, t=150, h=2, d=64, chunk 64
    gen = torch.Generator().manual_seed(0)
    b, t, h, d = 2, 150, 2, 64
    q = F.normalize(torch.randn(b, t, h, d, generator=gen), dim=-1) * d ** -0.5
    k = F.normalize(torch.randn(b, t, h, d, generator=gen), dim=-1)
    v = torch.randn(b, t, h, d, generator=gen)
    g = -torch.rand(b, t, h, generator=gen) * 0.2
    beta = torch.rand(b, t, h, generator=gen)
    s0 = torch.randn(b, h, d, d, generator=gen) * 0.1
    o, s = hk.delta_rule_reference(q, k, v, g, beta, 64, s0)
    out["gdn_prepare"] = dict(q=q, k=k, v=v, g=g, beta=beta, s0=s0, chunk=64, o=o, S=s)
    # D = 256, ragged T (not a chunk multiple), config-0 style inputs (bf16-valued q/k/v)
    torch.manual_seed(1)
    b, t, h, d = 1, 70, 1, 256
    q = bf(F.normalize(torch.randn(b, t, h, d), dim=-1))
    k = bf(F.normalize(torch.randn(b, t, h, d), dim=-1))
    v = bf(torch.randn(b, t, h, d))
    beta = torch.sigmoid(torch.randn(b, t, h))
    A_log = torch.empty(h).uniform_(-4, 0)
    g = -A_log.exp() * F.softplus(torch.randn(b, t, h))
    s0 = torch.randn(b, h, d, d) * 0.05
    o, s = hk.delta_rule_reference(q, k, v, g, beta, 64, s0)
    b16 = lambda z: z.to(torch.bfloat16)
    out["gdn_d256"] = dict(q=b16(q), k=b16(k), v=b16(v), g=g, beta=beta, s0=s0, chunk=64, o=o, S=s)
    # single recurrent step
    torch.manual_seed(2)
    b, h, d = 2, 3, 16
    q, k = torch.randn(b, h, d), F.normalize(torch.randn(b, h, d), dim=-1)
    v, g, beta, s0 = torch.randn(b, h, d), -torch.rand(b, h), torch.rand(b, h), torch.randn(b, h, d, d)
    o, s = hk.delta_rule_step(q, k, v, g, beta, s0)
    out["gdn_step"] = dict(q=q, k=k, v=v, g=g, beta=beta, s0=s0, o=o, S=s)
    # GQA form, shapes of tests/test_motor.py:28-39
    torch.manual_seed(0)
    B, T, G, R, D = 1, 77, 2, 3, 8
    q = torch.randn(B, T, G, R, D)
    k = F.normalize(torch.randn(B, T, G, D), dim=-1)
    v, g, beta = torch.randn(B, T, G, D), -torch.rand(B, T, G), torch.rand(B, T, G)
    s0 = torch.randn(B, G, D, D) * 0.1
    o, s = hm.delta_rule_gqa(q, k, v, g, beta, 16, s0)
    out["gdn_gqa"] = dict(q=q, k=k, v=v, g=g, beta=beta, s0=s0, chunk=16, o=o, S=s)
    return out


def layer_case(hb, name, H, G, D, d, window, sinks, archival, parts, seed, keep_window=False):
    """Run HybridAttention._student over ``parts`` (mixed prefill / decode) and once over the whole sequence."""
    a = hb.HybridAttention(hb.HybridConfig(module_config(H, G, D, d)))
    make_module_params(a, window, sinks, archival, seed)
    T = sum(parts)
    gen = torch.Generator().manual_seed(seed + 100)
    rms = lambda z: z * torch.rsqrt(z.square().mean(-1, keepdim=True) + 1e-6)
    x = bf(torch.randn(1, T, d, generator=gen))
    q = bf(rms(torch.randn(1, T, H, D, generator=gen)))
    k = bf(rms(torch.randn(1, T, G, D, generator=gen)))
    v = bf(rms(torch.randn(1, T, G, D, generator=gen)))
    # roped copies are independent inputs to _student; any bf16-valued tensors exercise the path
    qr = bf(rms(torch.randn(1, H, T, D, generator=gen)))
    kr = bf(rms(torch.randn(1, G, T, D, generator=gen)))
    with torch.no_grad():
        full = a._student(x, q, k, v, qr, kr, 0, None)
        cache, outs, s = {}, [], 0
        for n in parts:
            sl = slice(s, s + n)
            outs.append(a._student(x[:, sl], q[:, sl], k[:, sl], v[:, sl], qr[:, :, sl], kr[:, :, sl], s, cache))
            s += n
        o_win, lse = a._window(qr, torch.cat((kr.new_zeros(1, G, window, D), kr), 2),
                               torch.cat((v.new_zeros(1, G, window, D), v.transpose(1, 2)), 2),
                               torch.cat((torch.full((window,), -1, dtype=torch.long), torch.arange(T))),
                               kr[:, :, :min(sinks, T)], v.transpose(1, 2)[:, :, :min(sinks, T)], torch.arange(T))
    checks = {k_: float(p.detach().double().sum()) for k_, p in a.named_parameters() if k_.split(".")[0] in a.NEW}
    b16 = lambda z: z.to(torch.bfloat16)
    o_parts = torch.cat(outs, 1)
    rec = dict(H=H, G=G, D=D, d=d, window=window, sinks=sinks, archival=archival, seed=seed,
               parts=list(parts), x=b16(x), q=b16(q), k=b16(k), v=b16(v), qr=b16(qr), kr=b16(kr),
               o_parts=o_parts, full_vs_parts=float((full - o_parts).abs().max()),
               cache={k_: v_.clone() for k_, v_ in cache.items()}, lse=lse, param_sums=checks)
    if keep_window:
        rec["o_win"] = o_win
    return {name: rec}


def forward_case(hb, name, H, G, D, d, window, sinks, archival, parts, seed, mode="student"):
    """HybridAttention.forward of a converted layer (projections, ZNorm, partial RoPE, the core, the output gate
    and o_proj) over mixed prefill/decode ``parts``, in fp32 (the reference creates the converted layer's
    parameters in fp32) on bf16-valued inputs."""
    a = hb.HybridAttention(hb.HybridConfig(module_config(H, G, D, d)))
    make_module_params(a, window, sinks, archival, seed)
    make_module_proj(a, seed)
    a.mode = mode
    T = sum(parts)
    gen = torch.Generator().manual_seed(seed + 300)
    x = bf(torch.randn(1, T, d, generator=gen))
    with torch.no_grad():
        cache, outs, s = {}, [], 0
        for n in parts:
            outs.append(a.forward(x[:, s:s + n], cache, s))
            s += n
    return {name: dict(H=H, G=G, D=D, d=d, window=window, sinks=sinks, archival=archival, seed=seed, mode=mode,
                       rot=a.c.rot, theta=float(a.c.rope_theta), parts=list(parts), x=x,
                       y_parts=torch.cat(outs, 1), cache={k_: v_.clone() for k_, v_ in cache.items()})}


def gguf_case(proj):
    """The llama.cpp port's GGUF tensors of two converted layers, made by the reference's own
    ``tensors_from_conv`` (llamacpp/bifrost_gguf.py:23-44) from a conversion-parameter dict."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("bifrost_gguf", proj / "llamacpp" / "bifrost_gguf.py")
    bg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bg)
    names = {"fq": "fq", "fk": "fk", "ab_w": "ab.weight", "ab_b": "ab.bias", "mix_w": "mix.weight",
             "mix_b": "mix.bias", "mix_lse": "mix_lse", "mem_scale": "mem_scale", "A_log": "A_log",
             "dt_bias": "dt_bias"}
    conv, params, layers = [], {}, {}
    for i, (idx, archival) in enumerate(((3, 1), (7, 2))):
        p = param_tensors(4, 2, 32, 64, 16, archival, seed=10 + i)
        name = f"layers.{idx}"
        conv.append({"name": name, "archival": archival, "window": 16, "sinks": 4})
        for ours, theirs in names.items():
            params[f"{name}.self_attn.{theirs}"] = p[ours].clone()
        layers[idx] = p
    out, window, sinks = bg.tensors_from_conv({"conv": conv, "params": params})
    return {"layers": layers, "window": window, "sinks": sinks,
            "tensors": {i: {k: torch.from_numpy(v.copy()) for k, v in t.items()} for i, t in out.items()}}


def retrieval_case(hb):
    """The reference's retrieval mask (HybridAttention._retrieval_mask, hibrit.py:301-324) and the attention its
    _teacher computes with it (scaled_dot_product_attention with enable_gqa, hibrit.py:283-284), on seeded
    bf16-valued inputs: the test_hibrit.py shapes, a decode token at Bifrost head geometry and a prefill."""
    out = {}
    cases = [("small", 1, 4, 2, 8, 50, 3, dict(k=2, block=4, window=6, sinks=2)),
             ("decode_d256", 1, 24, 4, 256, 600, 1, dict(k=4, block=16, window=256, sinks=4)),
             ("prefill_d64", 1, 8, 2, 64, 700, 5, dict(k=3, block=32, window=128, sinks=4, prefill=True))]
    for i, (name, B, H, G, D, n, t, ret) in enumerate(cases):
        gen = torch.Generator().manual_seed(300 + i)
        qr = bf(torch.randn(B, H, t, D, generator=gen))
        kr = bf(torch.randn(B, G, n, D, generator=gen))
        vt = bf(torch.randn(B, G, n, D, generator=gen))
        mask = hb.HybridAttention._retrieval_mask(None, qr, kr, ret)
        o = F.scaled_dot_product_attention(qr, kr, vt, attn_mask=mask, enable_gqa=True).transpose(1, 2)
        b16 = lambda z: z.to(torch.bfloat16)   # bf16-valued: stored exactly in half the bytes
        out[name] = dict(qr=b16(qr), kr=b16(kr), vt=b16(vt), ret=ret, mask=mask, o=o)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("HEIMDALL_REFERENCE"))
    ap.add_argument("--cases", default="all", help="comma list of gdn, layer, forward, gguf, retrieval (default all)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("name the reference project with --ref or HEIMDALL_REFERENCE")
    ref = Path(args.ref)
    proj = ref / "Heimdall" if (ref / "Heimdall" / "heimdall").is_dir() else ref
    sys.path.insert(0, str(proj))
    import heimdall.hibrit as hb
    import heimdall.kernels as hk
    import heimdall.motor as hm
    torch.set_num_threads(8)
    cases = {"gdn", "layer", "forward", "gguf", "retrieval"} if args.cases == "all" else set(args.cases.split(","))
    if "gguf" in cases:
        torch.save(gguf_case(proj), HERE / "golden_gguf.pt")
    if "retrieval" in cases:
        torch.save(retrieval_case(hb), HERE / "golden_retrieval.pt")
    if "gdn" in cases:
        torch.save(gdn_cases(hk, hm), HERE / "golden_gdn.pt")
    layers = {}
    # tiny shapes of tests/test_hibrit.py (window 8, sinks 2, 4 Q / 2 KV heads, head_dim 32) with the
    # mixed prefill/decode part pattern of test_chunked_cache_equals_full
    layers.update(layer_case(hb, "tiny", H=4, G=2, D=32, d=64, window=8, sinks=2, archival=1,
                             parts=(5, 1, 13, 1, 1, 9, 30, 1), seed=0, keep_window=True))
    # Bifrost head geometry (24 Q / 4 KV, D=256, 4 sinks), short window so memory is active
    layers.update(layer_case(hb, "d256", H=24, G=4, D=256, d=128, window=16, sinks=4, archival=1,
                             parts=(10, 1, 13, 1, 5), seed=1))
    if "layer" in cases:
        torch.save(layers, HERE / "golden_layer.pt")
    fwd = {}
    # the whole converted attention layer in bf16 (the prologue and epilogue around the core), Bifrost heads
    fwd.update(forward_case(hb, "d256", H=24, G=4, D=256, d=64, window=16, sinks=4, archival=1,
                            parts=(21, 1, 9, 1), seed=2))
    fwd.update(forward_case(hb, "d256_window", H=24, G=4, D=256, d=64, window=16, sinks=4, archival=1,
                            parts=(30, 1), seed=3, mode="window"))
    if "forward" in cases:
        torch.save(fwd, HERE / "golden_forward.pt")
    meta = {"torch": torch.__version__,
            "reference": "Heimdall (heimdall.kernels / motor / hibrit incl. _retrieval_mask; llamacpp/bifrost_gguf.py)"}
    (HERE / "golden_meta.txt").write_text("\n".join(f"{k}: {v}" for k, v in meta.items()) + "\n")
    for f in sorted(HERE.glob("golden_*.pt")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()

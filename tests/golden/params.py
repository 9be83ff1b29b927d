"""Seeded layer parameters shared by the golden-fixture generator and the tests.

The fixtures store only checksums of these tensors; both the generator (which loads them into the
reference ``HybridAttention``) and the tests (which need them on machines without the reference)
rebuild them here from the seed with a private ``torch.Generator`` on the CPU.
"""
from __future__ import annotations

import math
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[2]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
from oracle.bifrost_oracle import LayerParams, ProjParams  # noqa: E402


def module_config(H: int, G: int, D: int, d: int) -> dict:
    """A Qwen3.5-style text config that the reference ``HybridConfig`` accepts, for one attention layer."""
    return dict(model_type="qwen3_5_text", vocab_size=300, hidden_size=d, intermediate_size=128,
                num_hidden_layers=4, num_attention_heads=H, num_key_value_heads=G, head_dim=D,
                linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=16,
                linear_value_head_dim=16, linear_conv_kernel_dim=4, full_attention_interval=4,
                attn_output_gate=True, rms_norm_eps=1e-6, hidden_act="silu",
                rope_parameters={"rope_type": "default", "rope_theta": 10000.0, "partial_rotary_factor": 0.25},
                tie_word_embeddings=False, mtp_num_hidden_layers=0, eos_token_id=0)


def param_tensors(H: int, G: int, D: int, d: int, window: int, archival: int, seed: int) -> dict:
    """Deterministic "as if trained" values: fq/fk near identity, non-zero gates, long-memory decay."""
    gen = torch.Generator().manual_seed(1000 + seed)
    n = lambda *s: torch.randn(*s, generator=gen)
    sd = 0.3 * math.sqrt(64.0 / d)
    dt = torch.exp(torch.empty(G).uniform_(math.log(1e-3), math.log(1e-1), generator=gen))
    life = torch.logspace(math.log10(max(window, 2)), 6.0, G)
    mask = torch.ones(G)
    mask[:archival] = 0.0
    return dict(fq=torch.eye(D).repeat(H, 1, 1) + 0.1 * n(H, D, D), fk=torch.eye(D).repeat(G, 1, 1) + 0.1 * n(G, D, D),
                ab_w=sd * n(2 * G, d), ab_b=0.3 * n(2 * G), mix_w=sd * n(H, d), mix_b=torch.full((H,), 0.5),
                mix_lse=0.5 * n(H), mem_scale=float(D) ** 0.5 + 0.1 * n(H),
                A_log=(math.log(2.0) / (life * dt)).log(), dt_bias=dt + torch.log(-torch.expm1(-dt)),
                decay_mask=mask)


def make_module_params(attn, window: int, sinks: int, archival: int, seed: int) -> None:
    """Convert a reference ``HybridAttention`` and overwrite its new parameters with ``param_tensors``."""
    c = attn.c
    attn.convert(window, sinks, archival, "long")
    p = param_tensors(c.h, c.hkv, c.dh, c.d, window, archival, seed)
    with torch.no_grad():
        attn.fq.copy_(p["fq"])
        attn.fk.copy_(p["fk"])
        attn.ab.weight.copy_(p["ab_w"])
        attn.ab.bias.copy_(p["ab_b"])
        attn.mix.weight.copy_(p["mix_w"])
        attn.mix.bias.copy_(p["mix_b"])
        attn.mix_lse.copy_(p["mix_lse"])
        attn.mem_scale.copy_(p["mem_scale"])
        attn.A_log.copy_(p["A_log"])
        attn.dt_bias.copy_(p["dt_bias"])
        attn.decay_mask.copy_(p["decay_mask"])


def layer_params(H: int, G: int, D: int, d: int, window: int, sinks: int, archival: int, seed: int) -> LayerParams:
    """The same values as an oracle ``LayerParams`` (no reference needed)."""
    return LayerParams(window=window, sinks=sinks, **param_tensors(H, G, D, d, window, archival, seed))


def proj_tensors(H: int, G: int, D: int, d: int, seed: int) -> dict:
    """Deterministic projection weights of one attention layer (q/gate, k, v, o, the two ZNorm weights), scaled
    so that the projections of unit-variance inputs have unit variance."""
    gen = torch.Generator().manual_seed(2000 + seed)
    n = lambda *s: torch.randn(*s, generator=gen)
    return dict(q_w=n(2 * H * D, d) * d ** -0.5, k_w=n(G * D, d) * d ** -0.5, v_w=n(G * D, d) * d ** -0.5,
                o_w=n(d, H * D) * (H * D) ** -0.5, q_norm_w=0.1 * n(D), k_norm_w=0.1 * n(D))


def make_module_proj(attn, seed: int) -> None:
    """Overwrite a reference ``HybridAttention``'s projections and norms with ``proj_tensors``."""
    c = attn.c
    t = proj_tensors(c.h, c.hkv, c.dh, c.d, seed)
    with torch.no_grad():
        attn.q_proj.weight.copy_(t["q_w"])
        attn.k_proj.weight.copy_(t["k_w"])
        attn.v_proj.weight.copy_(t["v_w"])
        attn.o_proj.weight.copy_(t["o_w"])
        attn.q_norm.weight.copy_(t["q_norm_w"])
        attn.k_norm.weight.copy_(t["k_norm_w"])


def proj_params(H: int, G: int, D: int, d: int, seed: int, rot: int, theta: float = 10000.0) -> ProjParams:
    """The same values as an oracle ``ProjParams`` (no reference needed)."""
    return ProjParams(rot=rot, theta=theta, **proj_tensors(H, G, D, d, seed))

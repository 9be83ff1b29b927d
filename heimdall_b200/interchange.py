"""Serving interchange with the reference's llama.cpp port: its per-sequence state row and its GGUF tensors.

State row (reference ``llamacpp/bifrost.patch``): every converted layer keeps one fp32 row per sequence in
llama.cpp's recurrent memory, ``llama_hparams::bifrost_state()`` floats long (bifrost.patch:221-239):
region [C, LR] of slot rows [k_rope | v | k_mem | g | beta], a K plane [D, LR, G], a transposed V plane
[LR, D, G] and the delta state [D, D, G] (key index fastest).  ``pack_llama_state`` turns this package's cache
dict (the reference's keys, ``heimdall/hibrit.py:414-423``) into those rows on the GPU and
``unpack_llama_state`` turns rows back into a cache, so a sequence prefilled here can be continued by a
llama.cpp server and the other way round.  Positions are not part of the row (llama.cpp keeps them in its
memory cells), so both take each sequence's next position.  The copies run in ``bf_llama_state_pack`` /
``bf_llama_state_unpack``; there is no CPU path.

GGUF tensors (reference ``llamacpp/bifrost_gguf.py:23-44``): ``gguf_tensors`` gives the per-layer tensors the
port loads (``blk.N.bifrost_fq`` ... ``bifrost_dt``) from a layer's parameters, ``gguf_metadata`` the
``<arch>.bifrost.*`` keys, and ``params_from_gguf`` the inverse, for building a ``BifrostLayer`` from a converted
GGUF.  These are one-time parameter reformats on the host (numpy arrays, ready for ``gguf.GGUFWriter``).
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib
from .functional import check_cuda, ptr, stream_handle
from .layer import PARAM_NAMES, BifrostLayer, ctypes_ref
from .structs import BfRingCache


def llama_state_floats(G: int, D: int, window: int, sinks: int) -> int:
    """Floats in one sequence's state row of one converted layer (llama_hparams::bifrost_state)."""
    n = _lib.size("bf_llama_state_floats", G, D, window, sinks)
    if n == 0:
        raise ValueError("bad state-row geometry")
    return n


def _next_pos(next_pos, B: int, dev) -> torch.Tensor:
    if isinstance(next_pos, int):
        return torch.full((B,), next_pos, dtype=torch.int64, device=dev)
    p = torch.as_tensor(next_pos).to(device=dev, dtype=torch.int64).contiguous().reshape(-1)
    if p.numel() != B:
        raise ValueError("next_pos must hold one position per sequence")
    return p


def _ring_struct(cache: dict, B: int, G: int, D: int, W: int, need_state: bool):
    bf = torch.bfloat16
    dev = cache["ring_k"].device
    shapes = {"ring_k": ((B, G, W, D), bf), "ring_v": ((B, G, W, D), bf), "ring_km": ((B, W, G, D), torch.float32),
              "ring_g": ((B, W, G), torch.float32), "ring_beta": ((B, W, G), torch.float32)}
    for key, (shape, dt) in shapes.items():
        t = cache[key]
        if tuple(t.shape) != shape or t.dtype != dt or not t.is_contiguous() or t.device != dev:
            raise ValueError(f"cache[{key!r}] must be a contiguous {dt} tensor {shape} on {dev}")
    rp = cache["ring_pos"]
    if rp.dtype != torch.int64 or not rp.is_contiguous() or not (rp.shape == (W,) or rp.shape == (B, W)):
        raise ValueError("cache['ring_pos'] must be a contiguous int64 [W] or [B, W]")
    sk, sv = cache.get("sink_k"), cache.get("sink_v")
    ns = 0 if sk is None else sk.shape[2]
    if sk is not None and (sk.dtype != bf or sv.dtype != bf or not sk.is_contiguous() or not sv.is_contiguous()
                           or tuple(sk.shape) != (B, G, ns, D) or tuple(sv.shape) != (B, G, ns, D)):
        raise ValueError("sinks must be contiguous bf16 [B, G, ns, D]")
    S = cache.get("S")
    if S is not None and (tuple(S.shape) != (B, G, D, D) or S.dtype != torch.float32 or not S.is_contiguous()):
        raise ValueError("cache['S'] must be a contiguous fp32 [B, G, D, D]")
    if need_state and S is None:
        raise ValueError("cache['S'] is required")
    return BfRingCache(ptr(cache["ring_k"]), ptr(cache["ring_v"]), ptr(cache["ring_km"]), ptr(cache["ring_g"]),
                       ptr(cache["ring_beta"]), ptr(rp), W if rp.dim() == 2 else 0, ptr(sk), ptr(sv), ns, ptr(S))


def pack_llama_state(layer: BifrostLayer, cache: dict, next_pos, rows=None) -> torch.Tensor:
    """The cache of B sequences (device tensors in kernel layout: ring_k/ring_v bf16, ring_pos [W] or [B,W],
    optional sinks and S) whose next positions are ``next_pos`` (int or [B]) -> rows [B, llama_state_floats]
    fp32 on the same device (or written into ``rows``, a [B, >= floats] fp32 tensor with unit inner stride)."""
    G, D, W, S = layer.G, layer.D, layer.window, layer.sinks
    check_cuda(cache["ring_k"])
    B = cache["ring_k"].shape[0]
    dev = cache["ring_k"].device
    n = llama_state_floats(G, D, W, S)
    if rows is None:
        rows = torch.empty(B, n, device=dev, dtype=torch.float32)
    if rows.dtype != torch.float32 or rows.dim() != 2 or rows.shape[0] != B or rows.shape[1] < n or rows.stride(1) != 1:
        raise ValueError("rows must be fp32 [B, >= llama_state_floats] with unit inner stride")
    rc = _ring_struct(cache, B, G, D, W, need_state=False)
    p = _next_pos(next_pos, B, dev)
    _lib.call("bf_llama_state_pack", ctypes_ref(rc), ptr(p), B, G, D, W, S, ptr(rows), rows.stride(0),
              stream_handle())
    return rows


def unpack_llama_state(layer: BifrostLayer, rows: torch.Tensor, next_pos, cache: dict | None = None,
                       per_seq_pos: bool = True) -> dict:
    """Rows [B, >= llama_state_floats] fp32 (device) of sequences at next positions ``next_pos`` -> a cache dict
    (written into ``cache`` when given, else allocated) with ring_pos [B, W] (``per_seq_pos``) or [W] (every
    sequence then at the same position) and min(sinks, next position) sink rows."""
    G, D, W, S = layer.G, layer.D, layer.window, layer.sinks
    check_cuda(rows)
    B = rows.shape[0]
    dev = rows.device
    n = llama_state_floats(G, D, W, S)
    if rows.dtype != torch.float32 or rows.dim() != 2 or rows.shape[1] < n or rows.stride(1) != 1:
        raise ValueError("rows must be fp32 [B, >= llama_state_floats] with unit inner stride")
    p = _next_pos(next_pos, B, dev)
    if cache is None:
        ns = int(min(S, int(p.min().item()))) if B else 0
        bf = torch.bfloat16
        cache = dict(ring_k=torch.empty(B, G, W, D, device=dev, dtype=bf),
                     ring_v=torch.empty(B, G, W, D, device=dev, dtype=bf),
                     ring_km=torch.empty(B, W, G, D, device=dev), ring_g=torch.empty(B, W, G, device=dev),
                     ring_beta=torch.empty(B, W, G, device=dev),
                     ring_pos=torch.empty((B, W) if per_seq_pos else (W,), device=dev, dtype=torch.int64),
                     sink_k=torch.empty(B, G, ns, D, device=dev, dtype=bf),
                     sink_v=torch.empty(B, G, ns, D, device=dev, dtype=bf),
                     S=torch.empty(B, G, D, D, device=dev))
        if ns == 0:
            cache["sink_k"] = cache["sink_v"] = None
    rc = _ring_struct(cache, B, G, D, W, need_state=True)
    _lib.call("bf_llama_state_unpack", ptr(rows), rows.stride(0), ptr(p), B, G, D, W, S, ctypes_ref(rc),
              stream_handle())
    return cache


# ------------------------------------------------------------------------------------------ GGUF tensors
GGUF_TENSORS = ("bifrost_fq", "bifrost_fk", "bifrost_ab", "bifrost_ab_b", "bifrost_mix", "bifrost_mix_b",
                "bifrost_mix_lse", "bifrost_mem_scale", "bifrost_a", "bifrost_dt")


def _host_params(src) -> dict:
    p = src.p if isinstance(src, BifrostLayer) else src
    return {n: torch.as_tensor(p[n]).detach().float().cpu() for n in PARAM_NAMES}


def gguf_tensors(src) -> dict:
    """A converted layer's GGUF tensors (bifrost_gguf.py:30-41), fp32 numpy arrays keyed by the names the port
    loads under ``blk.N.``: fq/fk with the two last axes swapped (so ggml's mul_mat applies q fq), the ab and
    mix linears, mix_lse, mem_scale, the decay rate a = -e^{A_log} decay_mask and dt_bias.  ``src``: a
    ``BifrostLayer`` or a dict with the names in ``PARAM_NAMES``."""
    p = _host_params(src)
    out = {"bifrost_fq": p["fq"].transpose(1, 2).contiguous(), "bifrost_fk": p["fk"].transpose(1, 2).contiguous(),
           "bifrost_ab": p["ab_w"], "bifrost_ab_b": p["ab_b"], "bifrost_mix": p["mix_w"], "bifrost_mix_b": p["mix_b"],
           "bifrost_mix_lse": p["mix_lse"], "bifrost_mem_scale": p["mem_scale"],
           "bifrost_a": -p["A_log"].exp() * p["decay_mask"], "bifrost_dt": p["dt_bias"]}
    return {k: v.numpy().astype(np.float32) for k, v in out.items()}


def gguf_metadata(window: int, sinks: int, bifrost_layers, n_block: int, arch: str = "qwen35") -> dict:
    """The ``<arch>.bifrost.*`` keys (bifrost_gguf.py:95-97): window, sinks and a 0/1 flag per block."""
    conv = set(int(i) for i in bifrost_layers)
    return {f"{arch}.bifrost.window": int(window), f"{arch}.bifrost.sinks": int(sinks),
            f"{arch}.bifrost.layers": [1 if i in conv else 0 for i in range(int(n_block))]}


def params_from_gguf(tensors: dict) -> dict:
    """The inverse of ``gguf_tensors``: a parameter dict for ``BifrostLayer``.  A head with a = 0 is archival
    (decay_mask 0); its A_log is not stored in the GGUF and is set to 0 (it is multiplied by the mask)."""
    t = {k: torch.as_tensor(np.asarray(v), dtype=torch.float32) for k, v in tensors.items()}
    a = t["bifrost_a"]
    mask = (a != 0).float()
    A_log = torch.where(a != 0, (-a).clamp_min(1e-30).log(), torch.zeros_like(a))
    return dict(fq=t["bifrost_fq"].transpose(1, 2).contiguous(), fk=t["bifrost_fk"].transpose(1, 2).contiguous(),
                ab_w=t["bifrost_ab"], ab_b=t["bifrost_ab_b"], mix_w=t["bifrost_mix"], mix_b=t["bifrost_mix_b"],
                mix_lse=t["bifrost_mix_lse"], mem_scale=t["bifrost_mem_scale"], A_log=A_log,
                dt_bias=t["bifrost_dt"], decay_mask=mask)

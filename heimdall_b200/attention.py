"""The whole converted attention layer on B200: the host mirror of ``HybridAttention.forward`` in student (or
window) mode (heimdall/hibrit.py:426-432): projections -> fused prologue -> the layer core -> fused epilogue ->
output projection.

The four projections are plain bf16 GEMMs on the GPU's GEMM library (cuBLAS through ``torch.nn.functional.linear``,
as the reference's ``nn.Linear`` layers run them).  Everything between them runs in this package's kernels:
``bf_attn_prologue`` (the per-head split of query and output gate, the ZNorm of q and k, the partial RoPE and the
two layouts the core reads, in one pass), the layer core (``BifrostLayer.student``), and ``bf_attn_epilogue``
(the output gate o * sigmoid(gate) in bf16, ready for o_proj).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import _lib
from .functional import check_cuda, ptr, stream_handle
from .layer import BifrostLayer


class BifrostAttention:
    """A converted attention layer's projections and core on one CUDA device.

    ``q_w`` [H*D*(2 if gated else 1), d] (query and output gate interleaved per head, as Qwen3.5's q_proj),
    ``k_w``/``v_w`` [G*D, d], ``o_w`` [d, H*D], optional biases, ``q_norm_w``/``k_norm_w`` [D] (zero-centred
    ZNorm weights), RoPE on the first ``rot`` dims with base ``theta``, norm ``eps``; ``layer`` the converted
    core (``BifrostLayer``).  ``mode``: "student" (window + memory) or "window" (the reference's memoryless mode).
    """

    def __init__(self, q_w, k_w, v_w, o_w, q_norm_w, k_norm_w, layer: BifrostLayer, rot: int, theta: float,
                 eps: float = 1e-6, gated: bool = True, q_b=None, k_b=None, v_b=None, o_b=None, mode: str = "student"):
        dev = layer.device
        bf = torch.bfloat16
        cvt = lambda t: None if t is None else t.detach().to(device=dev, dtype=bf).contiguous()
        self.q_w, self.k_w, self.v_w, self.o_w = cvt(q_w), cvt(k_w), cvt(v_w), cvt(o_w)
        self.q_b, self.k_b, self.v_b, self.o_b = cvt(q_b), cvt(k_b), cvt(v_b), cvt(o_b)
        f32 = lambda t: t.detach().to(device=dev, dtype=torch.float32).contiguous()
        self.q_norm_w, self.k_norm_w = f32(q_norm_w), f32(k_norm_w)
        self.layer, self.rot, self.theta, self.eps, self.gated = layer, int(rot), float(theta), float(eps), bool(gated)
        if mode not in ("student", "window"):
            raise ValueError("mode must be 'student' or 'window'")
        self.mode = mode
        H, G, D = layer.H, layer.G, layer.D
        if tuple(self.q_w.shape) != (H * D * (2 if gated else 1), layer.d) or tuple(self.k_w.shape) != (G * D, layer.d):
            raise ValueError("projection shapes do not match the layer")
        # inverse RoPE frequencies exactly as the reference computes them (heimdall/kernels.py:44), in fp32
        d_rot = max(self.rot, 2)
        self.inv_freq = (1.0 / (self.theta ** (torch.arange(0, d_rot, 2, dtype=torch.float32) / d_rot))).to(dev)

    @classmethod
    def from_module(cls, attn, device=None) -> "BifrostAttention":
        """From a converted reference ``HybridAttention`` (its projections, norms, RoPE config and new parameters)."""
        c = attn.c
        layer = BifrostLayer.from_module(attn, device)
        bias = lambda lin: None if lin.bias is None else lin.bias
        return cls(attn.q_proj.weight, attn.k_proj.weight, attn.v_proj.weight, attn.o_proj.weight,
                   attn.q_norm.weight, attn.k_norm.weight, layer, c.rot, c.rope_theta, c.eps, c.gate,
                   bias(attn.q_proj), bias(attn.k_proj), bias(attn.v_proj), bias(attn.o_proj),
                   mode="window" if attn.mode == "window" else "student")

    def project(self, x, start: int = 0):
        """``HybridAttention._proj`` (heimdall/hibrit.py:254-268): x [B,t,d] -> (q, k, v, qr, kr, qg) with q
        [B,t,H,D], k/v [B,t,G,D] (ZNorm'd), qr [B,H,t,D], kr [B,G,t,D] (partial RoPE) in bf16, and qg the query
        projection [B,t,H,(2 if gated) D] holding the output gate."""
        check_cuda(x)
        L = self.layer
        B, t = x.shape[:2]
        H, G, D = L.H, L.G, L.D
        xb = x.to(torch.bfloat16)
        qg = F.linear(xb, self.q_w, self.q_b).contiguous()
        kl = F.linear(xb, self.k_w, self.k_b).contiguous()
        v = F.linear(xb, self.v_w, self.v_b).view(B, t, G, D)
        dev = x.device
        q = torch.empty(B, t, H, D, device=dev, dtype=torch.bfloat16)
        k = torch.empty(B, t, G, D, device=dev, dtype=torch.bfloat16)
        qr = torch.empty(B, H, t, D, device=dev, dtype=torch.bfloat16)
        kr = torch.empty(B, G, t, D, device=dev, dtype=torch.bfloat16)
        _lib.call("bf_attn_prologue", ptr(qg), ptr(kl), ptr(self.q_norm_w), ptr(self.k_norm_w),
                  ptr(self.inv_freq) if self.rot else None, self.rot, self.eps, int(start), None, B, t, H, G, D,
                  1 if self.gated else 0, ptr(q), ptr(k), ptr(qr), ptr(kr), stream_handle())
        return q, k, v.contiguous(), qr, kr, qg

    def output(self, o, qg, x):
        """``HybridAttention._out`` (heimdall/hibrit.py:270-272): o [B,t,H,D] fp32 -> o_proj(o * sigmoid(gate))."""
        L = self.layer
        B, t = x.shape[:2]
        y = torch.empty(B, t, L.H * L.D, device=x.device, dtype=torch.bfloat16)
        _lib.call("bf_attn_epilogue", ptr(o.contiguous()), ptr(qg), 1 if self.gated else 0, B, t, L.H, L.D, ptr(y),
                  stream_handle())
        return F.linear(y, self.o_w, self.o_b)

    def forward(self, x, cache=None, start: int = 0):
        """``HybridAttention.forward`` of a converted layer (heimdall/hibrit.py:426-432): x [B,t,d] -> [B,t,d] bf16,
        with the reference's cache dict (prefill for t > 1, the decode step for t == 1 with a cache)."""
        q, k, v, qr, kr, qg = self.project(x, start)
        o = self.layer.student(x, q, k, v, qr, kr, int(start), cache, memory=self.mode != "window")
        o = o.reshape(*x.shape[:2], self.layer.H, self.layer.D)
        return self.output(o, qg, x)

    __call__ = forward

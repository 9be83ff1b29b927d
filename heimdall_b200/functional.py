"""Tensor-level wrappers of the C ABI with the reference's function signatures.

Each wrapper mirrors a function of the reference package ``heimdall`` (argument names, shapes,
fp32 outputs, exceptions) and runs only on CUDA tensors: there is no CPU fallback.  Inputs are
made contiguous; q/k/v may be fp32 or bf16 where the kernel accepts both.
"""
from __future__ import annotations

import torch

from . import _lib


def check_cuda(*ts) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("heimdall_b200 runs on CUDA tensors only (there is no CPU fallback)")


def stream_handle() -> int:
    return torch.cuda.current_stream().cuda_stream


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def delta_rule_step(q, k, v, g, beta, state):
    """One recurrent gated delta-rule token (mirror of ``heimdall.kernels.delta_rule_step``, kernels.py:132-138).

    q, k: [B,H,Dk]; v: [B,H,Dv]; g, beta: [B,H]; state: [B,H,Dk,Dv].  Returns (o [B,H,Dv] fp32, new state fp32).
    The state is square here (Dk == Dv), as in the Bifrost layer.
    """
    check_cuda(q, k, v, g, beta, state)
    B, H, Dk = k.shape
    Dv = v.shape[-1]
    if Dk != Dv or tuple(state.shape) != (B, H, Dk, Dv):
        raise NotImplementedError("heimdall_b200 implements square states [B,H,D,D]")
    q32 = q.float().contiguous()
    k32 = k.float().contiguous()
    vv = v.contiguous() if v.dtype == torch.bfloat16 else v.float().contiguous()
    g32 = g.float().contiguous()
    b32 = beta.float().contiguous()
    s_in = state.float().contiguous()
    s_out = torch.empty_like(s_in)
    o = torch.empty(B, H, Dv, device=q.device, dtype=torch.float32)
    _lib.call("bf_gdn_decode_step", ptr(q32), ptr(k32), ptr(vv), 1 if vv.dtype == torch.bfloat16 else 0, ptr(g32),
              ptr(b32), ptr(s_in), ptr(s_out), ptr(o), B, H, 1, Dk, stream_handle())
    return o, s_out


def delta_rule_step_gqa(q, k, v, g, beta, state, out_state=None):
    """GQA form of one decode step: q [B,G,R,D], k/v [B,G,D], g/beta [B,G], state [B,G,D,D].

    This is the inline update of ``HybridAttention._student`` for t == 1 (hibrit.py:398-403).
    ``out_state`` may be ``state`` itself (in-place update).  Returns (o [B,G,R,D], new state).
    """
    check_cuda(q, k, v, g, beta, state)
    B, G, R, D = q.shape
    q32, k32 = q.float().contiguous(), k.float().contiguous()
    vv = v.contiguous() if v.dtype == torch.bfloat16 else v.float().contiguous()
    s_in = state if (state.dtype == torch.float32 and state.is_contiguous()) else state.float().contiguous()
    s_out = torch.empty_like(s_in) if out_state is None else out_state
    o = torch.empty(B, G, R, D, device=q.device, dtype=torch.float32)
    _lib.call("bf_gdn_decode_step", ptr(q32), ptr(k32), ptr(vv), 1 if vv.dtype == torch.bfloat16 else 0,
              ptr(g.float().contiguous()), ptr(beta.float().contiguous()), ptr(s_in), ptr(s_out), ptr(o),
              B, G, R, D, stream_handle())
    return o, s_out

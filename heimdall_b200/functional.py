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


def _ws(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)


def _dt(t) -> int:
    return 1 if t.dtype == torch.bfloat16 else 0


def _as_kernel_dtype(t):
    return t.contiguous() if t.dtype == torch.bfloat16 else t.float().contiguous()


def delta_rule_gqa(q, k, v, g, beta, chunk: int = 64, state=None, cu_seqlens=None):
    """GQA-native chunked gated delta rule (mirror of ``heimdall.motor.delta_rule_gqa``, motor.py:70-102).

    q [B,T,G,R,Dk]; k [B,T,G,Dk]; v [B,T,G,Dv]; g, beta [B,T,G]; state [B,G,Dk,Dv] or None.
    Returns o [B,T,G,R,Dv] and the final state [B,G,Dk,Dv], both fp32.  ``chunk`` is accepted for signature
    compatibility: the GPU scan always uses 128-token chunks (the recurrence, hence the result, does not
    depend on the chunk length).
    ``cu_seqlens`` (int tensor [n+1], cumulative lengths, B = 1): the T tokens are n packed sequences, each
    with its own recurrence; state and the returned final states are then [n,G,Dk,Dv].
    Differentiable (as the reference's torch ops are, which seq_loss, motor.py:149-193, trains through): with
    grad mode on and an input that requires grad, the backward runs ``bf_gdn_bwd`` (fp32, all six inputs).
    """
    check_cuda(q, k, v, g, beta, state, cu_seqlens)
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in (q, k, v, g, beta, state)):
        if cu_seqlens is not None:
            raise NotImplementedError("heimdall_b200: the delta-rule backward takes unpacked sequences (no cu_seqlens)")
        return _DeltaRuleGQA.apply(q, k, v, g, beta, state)
    return _delta_rule_gqa_fwd(q, k, v, g, beta, state, cu_seqlens)


def _delta_rule_gqa_fwd(q, k, v, g, beta, state, cu_seqlens):
    B, T, G, R, D = q.shape
    if k.shape[-1] != D or v.shape[-1] != D:
        raise NotImplementedError("heimdall_b200 implements square states (Dk == Dv)")
    if D != 256:
        raise NotImplementedError("the tensor-core delta rule is built for head dim 256")
    n_seq = 0
    cu = None
    if cu_seqlens is not None:
        if B != 1:
            raise ValueError("packed sequences (cu_seqlens) need batch size 1")
        cu = cu_seqlens.to(device=q.device, dtype=torch.int32).contiguous()
        n_seq = cu.numel() - 1
        if n_seq <= 0:
            raise ValueError("cu_seqlens needs at least two entries")
    dev = q.device
    qq, kk, vv = _as_kernel_dtype(q), _as_kernel_dtype(k), _as_kernel_dtype(v)
    gg, bb = g.float().contiguous(), beta.float().contiguous()
    s0 = None if state is None else state.float().contiguous()
    o = torch.empty(B, T, G, R, D, device=dev, dtype=torch.float32)
    s_out = torch.empty(n_seq if n_seq else B, G, D, D, device=dev, dtype=torch.float32)
    nws = _lib.size("bf_gdn_chunk_workspace", B, T, G, R, D, n_seq)
    ws = _ws(nws, dev)
    _lib.call("bf_gdn_chunk_fwd", ptr(qq), _dt(qq), ptr(kk), _dt(kk), ptr(vv), _dt(vv), ptr(gg), ptr(bb), ptr(s0),
              ptr(o), ptr(s_out), ptr(cu), n_seq, B, T, G, R, D, ptr(ws), nws, stream_handle())
    return o, s_out


def delta_rule_gqa_backward(q, k, v, g, beta, state, do, dstate):
    """Gradients of ``delta_rule_gqa`` (B sequences of T tokens): (dq, dk, dv, dg, dbeta, dstate0), all fp32 in the
    inputs' shapes; ``do`` = dL/do [B,T,G,R,D] and ``dstate`` = dL/d(final state) [B,G,D,D], either may be None
    (zero).  The torch autograd of motor.py:70-102 as seq_loss (motor.py:149-193) takes it, on ``bf_gdn_bwd``."""
    check_cuda(q, k, v, g, beta, state, do, dstate)
    B, T, G, R, D = q.shape
    if D != 256 or k.shape[-1] != D or v.shape[-1] != D:
        raise NotImplementedError("the delta-rule backward is built for head dim 256")
    dev = q.device
    f = lambda t: None if t is None else t.float().contiguous()
    qq, kk, vv, gg, bb, s0, dd, dst = (f(t) for t in (q, k, v, g, beta, state, do, dstate))
    if dd is None:
        dd = torch.zeros(B, T, G, R, D, device=dev)
    dq, dk, dv = torch.empty_like(qq), torch.empty_like(kk), torch.empty_like(vv)
    dg, db = torch.empty_like(gg), torch.empty_like(bb)
    ds0 = torch.empty(B, G, D, D, device=dev)
    nws = _lib.size("bf_gdn_bwd_workspace", B, T, G, R, D)
    ws = _ws(nws, dev)
    _lib.call("bf_gdn_bwd", ptr(qq), ptr(kk), ptr(vv), ptr(gg), ptr(bb), ptr(s0), ptr(dd), ptr(dst), ptr(dq), ptr(dk),
              ptr(dv), ptr(dg), ptr(db), ptr(ds0), B, T, G, R, D, ptr(ws), nws, stream_handle())
    return dq, dk, dv, dg, db, ds0


class _DeltaRuleGQA(torch.autograd.Function):
    """delta_rule_gqa with its backward on the GPU: forward on the chunked tensor-core scan, backward on
    ``bf_gdn_bwd`` from the saved inputs (the states are recomputed, none is kept)."""

    @staticmethod
    def forward(ctx, q, k, v, g, beta, state):
        o, s = _delta_rule_gqa_fwd(q, k, v, g, beta, state, None)
        ctx.save_for_backward(q, k, v, g, beta, state)
        return o, s

    @staticmethod
    def backward(ctx, do, dstate):
        q, k, v, g, beta, state = ctx.saved_tensors
        dq, dk, dv, dg, db, ds0 = delta_rule_gqa_backward(q, k, v, g, beta, state, do, dstate)
        return (dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), dg.to(g.dtype), db.to(beta.dtype),
                None if state is None else ds0.to(state.dtype))


def delta_rule(q, k, v, g, beta, chunk_size: int = 64, initial_state=None, backend: str = "auto", cu_seqlens=None):
    """Chunked gated delta rule (mirror of ``heimdall.kernels.delta_rule``, kernels.py:94-129 / 152-155).

    q, k: [B,T,H,Dk]; v: [B,T,H,Dv]; g, beta: [B,T,H]; initial_state [B,H,Dk,Dv] or None.
    Returns o [B,T,H,Dv] and the final state [B,H,Dk,Dv] (fp32).  ``backend`` is accepted for signature
    compatibility; this implementation always runs the CUDA kernels (there is no CPU path).
    ``cu_seqlens``: packed sequences as in ``delta_rule_gqa`` (states [n,H,Dk,Dv]).
    """
    B, T, H, D = q.shape
    o, s = delta_rule_gqa(q.reshape(B, T, H, 1, D), k, v, g, beta, chunk_size, initial_state, cu_seqlens)
    return o.reshape(B, T, H, D), s


def window_attention(qr, ext_k, ext_v, qpos0: int, kpos0: int, klo: int, window: int, sink_k=None, sink_v=None,
                     with_lse: bool = True):
    """Sliding-window + sink attention (the math of ``HybridAttention._window_fp32``, hibrit.py:341-361).

    qr [B,H,Tq,D] (query i at position qpos0 + i); ext_k [B,G,Tk,D] and ext_v [B,G,Tk,D] or any strided view
    (key j at position kpos0 + j); keys with position < klo are not window keys; sink_k/sink_v [B,G,ns,D]
    (positions 0..ns-1) or None.  Returns o [B,Tq,H,D] and lse [B,H,Tq] (fp32).
    """
    check_cuda(qr, ext_k, ext_v, sink_k, sink_v)
    B, H, Tq, D = qr.shape
    G, Tk = ext_k.shape[1], ext_k.shape[2]
    bf = torch.bfloat16
    qb = qr.to(bf).contiguous()
    kb = ext_k.to(bf).contiguous()
    vb = ext_v.to(bf)
    if vb.stride(-1) != 1:
        vb = vb.contiguous()
    ns = 0 if sink_k is None else sink_k.shape[2]
    skb = None if sink_k is None else sink_k.to(bf).contiguous()
    svb = None if sink_v is None else sink_v.to(bf).contiguous()
    o = torch.empty(B, Tq, H, D, device=qr.device, dtype=torch.float32)
    lse = torch.empty(B, H, Tq, device=qr.device, dtype=torch.float32) if with_lse else None
    nws = _lib.size("bf_window_workspace", B, G, Tk, D)
    ws = _ws(nws, qr.device)
    _lib.call("bf_window_attn_fwd", ptr(qb), ptr(kb), ptr(vb), vb.stride(0), vb.stride(1), vb.stride(2), ptr(skb),
              ptr(svb), ns, int(qpos0), int(kpos0), int(klo), B, H, G, Tq, Tk, D, int(window), ptr(o), ptr(lse),
              ptr(ws), nws, stream_handle())
    return o, lse


def segment_transform(k, v, g, beta, s0=None):
    """State map of one segment of the write stream, for sequence parallelism of the delta rule.

    k, v [B,T,G,D] (fp32 or bf16), g, beta [B,T,G], s0 [B,G,D,D] or None.  Returns (M, N), both
    [B,G,D,D] fp32: N is the final state of ``delta_rule_gqa`` over the segment from s0 (zero state when
    None), and for any other initial state S the final state is M (S - s0) + N.  The reference runs the
    same recurrence as one sequential scan (heimdall/kernels.py:118-129).
    """
    check_cuda(k, v, g, beta, s0)
    B, T, G, D = k.shape
    if D != 256 or v.shape[-1] != D:
        raise NotImplementedError("the tensor-core delta rule is built for head dim 256")
    dev = k.device
    kk, vv = _as_kernel_dtype(k), _as_kernel_dtype(v)
    gg, bb = g.float().contiguous(), beta.float().contiguous()
    s0c = None if s0 is None else s0.float().contiguous()
    M = torch.empty(B, G, D, D, device=dev, dtype=torch.float32)
    N = torch.empty(B, G, D, D, device=dev, dtype=torch.float32)
    nws = _lib.size("bf_gdn_segment_workspace", B, T, G, D)
    ws = _ws(nws, dev)
    _lib.call("bf_gdn_segment_transform", ptr(kk), _dt(kk), ptr(vv), _dt(vv), ptr(gg), ptr(bb), ptr(s0c), ptr(M),
              ptr(N), B, T, G, D, ptr(ws), nws, stream_handle())
    return M, N


def apply_prefix(M, N, s0=None):
    """Incoming states of consecutive segments: M, N [n,B,G,D,D] (segments in order), s0 [B,G,D,D] or None.
    Returns S [n+1,B,G,D,D] fp32 with S[0] = s0 (zero state when None) and S[j+1] = M[j] S[j] + N[j]."""
    check_cuda(M, N, s0)
    n, B, G, D = M.shape[0], M.shape[1], M.shape[2], M.shape[3]
    Mc, Nc = M.float().contiguous(), N.float().contiguous()
    s0c = None if s0 is None else s0.float().contiguous()
    S = torch.empty(n + 1, B, G, D, D, device=M.device, dtype=torch.float32)
    _lib.call("bf_gdn_apply_prefix", ptr(Mc), ptr(Nc), n, ptr(s0c), ptr(S), B, G, D, stream_handle())
    return S

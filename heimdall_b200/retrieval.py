"""Kept (not converted) full-attention layers on B200: ``HybridAttention._teacher`` with its retrieval branch
(heimdall/hibrit.py:275-324).

``teacher(qr, kr, v, cache, retrieval)`` has the reference's signature and cache semantics: the cache dict's
"k" and "v" hold every key and value so far ([B,G,n,D], kr's dtype).  Here they are views of capacity buffers
that grow geometrically (the reference concatenates the whole cache every call), and the cache also keeps the
per-block key min / max of the retrieval summaries, updated for each block that fills.  A single-token decode
with retrieval on and enough history (n - sinks - window >= k * block) runs ``bf_ret_decode`` (block bounds from
the summaries, top-k selection, exact attention over sinks + selected blocks + window); every other call is
causal attention over the whole cache on the window kernel (``bf_window_attn_fwd`` with the window as long as
the sequence).  Retrieval in prefill (``prefill=True`` with t > 1, a different selection per query) is not
built and raises.  There is no CPU path.
"""
from __future__ import annotations

import torch

from . import _lib
from .functional import check_cuda, ptr, stream_handle, window_attention


def _grow(cache: dict, B: int, G: int, D: int, n_new: int, dev, dtype, block: int) -> None:
    cap = cache.get("_cap", 0)
    if n_new <= cap:
        return
    new_cap = max(1024, 1 << (max(n_new, 1) - 1).bit_length())
    kb = torch.empty(B, G, new_cap, D, device=dev, dtype=dtype)
    vb = torch.empty(B, G, new_cap, D, device=dev, dtype=dtype)
    n = cache.get("_n", 0)
    if n:
        kb[:, :, :n].copy_(cache["k"])
        vb[:, :, :n].copy_(cache["v"])
    nbcap = new_cap // block
    kmin = torch.empty(B, G, nbcap, D, device=dev, dtype=dtype)
    kmax = torch.empty(B, G, nbcap, D, device=dev, dtype=dtype)
    nb = cache.get("_ret_nb", 0)
    if nb and cache.get("_ret_block") == block:
        kmin[:, :, :nb].copy_(cache["_ret_kmin"][:, :, :nb])
        kmax[:, :, :nb].copy_(cache["_ret_kmax"][:, :, :nb])
    else:
        nb = 0
    cache.update(_kbuf=kb, _vbuf=vb, _cap=new_cap, _ret_kmin=kmin, _ret_kmax=kmax, _ret_nb=nb, _ret_block=block)


def teacher(qr, kr, v, cache=None, retrieval=None):
    """HybridAttention._teacher (hibrit.py:275-290): qr [B,H,t,D], kr [B,G,t,D], v [B,t,G,D] (bf16 on CUDA) ->
    o [B,t,H,D] in qr's dtype.  ``cache`` (or None) keeps "k", "v" [B,G,n,D]; ``retrieval`` is the dict that
    ``set_retrieval`` stores (k, block, window, sinks, prefill) or None."""
    check_cuda(qr, kr, v)
    B, H, t, D = qr.shape
    G = kr.shape[1]
    dev, bf = qr.device, torch.bfloat16
    vt = v.transpose(1, 2)
    ret = retrieval
    block = int(ret["block"]) if ret is not None else 64
    if cache is None:
        k_all, v_all, n = kr.to(bf), vt.to(bf), t
    else:
        if "k" in cache and "_kbuf" not in cache:       # a cache the reference built: adopt its tensors
            k0, v0 = cache["k"], cache["v"]
            cache["_n"] = 0
            _grow(cache, B, G, D, k0.shape[2], dev, bf, block)
            cache["_kbuf"][:, :, :k0.shape[2]].copy_(k0)
            cache["_vbuf"][:, :, :k0.shape[2]].copy_(v0)
            cache["_n"] = k0.shape[2]
        n0 = cache.get("_n", 0)
        n = n0 + t
        _grow(cache, B, G, D, n, dev, bf, block)
        cache["_kbuf"][:, :, n0:n].copy_(kr)
        cache["_vbuf"][:, :, n0:n].copy_(vt)
        cache["_n"] = n
        cache["k"], cache["v"] = cache["_kbuf"][:, :, :n], cache["_vbuf"][:, :, :n]
        k_all, v_all = cache["k"], cache["v"]
    use_ret = ret is not None and (t == 1 or ret.get("prefill")) and \
        n - ret["sinks"] - ret["window"] >= ret["k"] * ret["block"]
    if use_ret and t > 1:
        raise NotImplementedError("heimdall_b200 retrieval: prefill with retrieval (a selection per query) "
                                  "is not built; the decode path is")
    if not use_ret:
        # causal attention over the whole cache: the window kernel with the window as long as the sequence
        o, _ = window_attention(qr, k_all.contiguous(), v_all, n - t, 0, 0, max(n, 1), None, None, with_lse=False)
        return o.to(qr.dtype)
    S, W, L, K = int(ret["sinks"]), int(ret["window"]), int(ret["block"]), int(ret["k"])
    if cache is None:           # one-off call: summaries of this cache only
        cache = {}
        _grow(cache, B, G, D, n, dev, bf, L)
        cache["_kbuf"][:, :, :n].copy_(k_all)
        cache["_vbuf"][:, :, :n].copy_(v_all)
    if cache.get("_ret_block") != L:
        cache.update(_ret_block=L, _ret_nb=0, _ret_kmin=torch.empty(B, G, cache["_cap"] // L, D, device=dev, dtype=bf),
                     _ret_kmax=torch.empty(B, G, cache["_cap"] // L, D, device=dev, dtype=bf))
    cap = cache["_cap"]
    nbcap = cache["_ret_kmin"].shape[2]
    nb_full = (n - S) // L
    nb0 = cache["_ret_nb"]
    if nb_full > nb0:
        _lib.call("bf_ret_summarize", ptr(cache["_kbuf"]), cap, B, G, D, S, L, nb0, nb_full, ptr(cache["_ret_kmin"]),
                  ptr(cache["_ret_kmax"]), nbcap, stream_handle())
        cache["_ret_nb"] = nb_full
    q = qr.reshape(B, H, D).to(bf).contiguous()
    o = torch.empty(B, H, D, device=dev, dtype=torch.float32)
    nws = _lib.size("bf_ret_decode_workspace", B, H, G, D, n, S, W, L, K)
    ws = torch.empty(nws, dtype=torch.uint8, device=dev)
    _lib.call("bf_ret_decode", ptr(q), ptr(cache["_kbuf"]), ptr(cache["_vbuf"]), cap, ptr(cache["_ret_kmin"]),
              ptr(cache["_ret_kmax"]), nbcap, B, H, G, D, n, S, W, L, K, ptr(o), ptr(ws), nws, stream_handle())
    return o.reshape(B, 1, H, D).to(qr.dtype)

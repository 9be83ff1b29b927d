"""Drop-in installation into the reference package, following its ``kernels.prepare`` plug-in convention.

Heimdall picks its fast delta-rule kernel in ``heimdall.kernels.prepare(device, backend)``
(heimdall/kernels.py:158-188): a candidate is self-tested against ``delta_rule_reference`` on seeded data
and enabled only when the relative error (outputs and final state) is below 0.03.  ``motor`` imports its op
by value (heimdall/motor.py:37), so the patch points are that module attribute and the ``HybridAttention``
methods that implement the converted (Bifrost) layer core:

  heimdall.motor.delta_rule_gqa                   (motor.py:70-102)     -> functional.delta_rule_gqa
  heimdall.motor.window_attention                 (motor.py:105-115)    -> functional.window_attention
  HybridAttention._student                        (hibrit.py:363-424)   -> BifrostLayer.student
  HybridAttention._window                         (hibrit.py:336-361)   -> functional.window_attention
  HybridAttention._mem_inputs                     (hibrit.py:327-334)   -> BifrostLayer.mem_inputs
  HybridAttention._teacher                        (hibrit.py:275-290)   -> retrieval.teacher (kept layers: causal
                                                                           attention, retrieval decode)

The module-level ``delta_rule`` / ``delta_rule_step`` of ``heimdall.kernels`` and their by-value copies in
``heimdall.hibrit`` (hibrit.py:32) are deliberately left alone: the model's linear-attention layers (Qwen3.5
Gated DeltaNet, hibrit.py:170-180) call them with their own head sizes, which these head-dim-256 kernels do
not cover, and the Bifrost layer never reaches them once ``_student`` is replaced.  The wrappers
``delta_rule`` and ``delta_rule_step`` below are still exported for callers that want the B200 ops by name.

``prepare(device, backend="b200")`` runs the reference's self-test shape (seeded q, k, v, g, beta and an
initial state, head dim 256 because the kernels are built for it) against the host package's
``delta_rule_reference`` and installs the patches.  Two deliberate differences from the reference: a failed
self-test raises instead of falling back, and the patched functions raise on CPU tensors (there is no CPU
path in this package).  ``uninstall()`` restores the originals.
"""
from __future__ import annotations

import importlib

import torch

from . import functional as F_
from . import retrieval as R_
from .layer import BifrostLayer

_SAVED: list = []          # (owner, attribute name, original value) in patch order
# what install() replaces: (module key, attribute path)
PATCHED_NAMES = (("motor", "delta_rule_gqa"), ("motor", "window_attention"), ("hibrit", "HybridAttention._student"),
                 ("hibrit", "HybridAttention._mem_inputs"), ("hibrit", "HybridAttention._window"),
                 ("hibrit", "HybridAttention._teacher"))
SELF_TEST_TOL = 0.03       # the reference's acceptance threshold (kernels.py:182)


def _modules(modules):
    if modules is not None:
        return modules
    return {name: importlib.import_module(f"heimdall.{name}") for name in ("kernels", "hibrit", "motor")}


def _patch(owner, name, value):
    if not hasattr(owner, name):
        raise AttributeError(f"{owner!r} has no attribute {name!r} to replace")
    _SAVED.append((owner, name, getattr(owner, name)))
    setattr(owner, name, value)


def _require_cuda(*ts):
    for t in ts:
        if isinstance(t, torch.Tensor) and not t.is_cuda:
            raise RuntimeError("heimdall_b200 is installed: the Bifrost path runs on CUDA tensors only")


# ---------------------------------------------------------------------------------------------- op wrappers
def delta_rule(q, k, v, g, beta, chunk_size: int = 64, initial_state=None, backend: str = "auto"):
    """heimdall.kernels.delta_rule (kernels.py:152-155) on the B200 kernels."""
    _require_cuda(q, k, v, g, beta, initial_state)
    return F_.delta_rule(q, k, v, g, beta, chunk_size, initial_state, backend)


def delta_rule_step(q, k, v, g, beta, state):
    """heimdall.kernels.delta_rule_step (kernels.py:132-138) on the B200 kernels."""
    _require_cuda(q, k, v, g, beta, state)
    return F_.delta_rule_step(q, k, v, g, beta, state)


def delta_rule_gqa(q, k, v, g, beta, chunk: int = 64, state=None):
    """heimdall.motor.delta_rule_gqa (motor.py:70-102) on the B200 kernels."""
    _require_cuda(q, k, v, g, beta, state)
    return F_.delta_rule_gqa(q, k, v, g, beta, chunk, state)


# ---------------------------------------------------------------------------------------------- module methods
_LAYER_ATTRS = ("fq", "fk", "A_log", "dt_bias", "mix_lse", "mem_scale", "decay_mask")


def _layer_key(attn, device):
    ts = [getattr(attn, n) for n in _LAYER_ATTRS] + [attn.ab.weight, attn.ab.bias, attn.mix.weight, attn.mix.bias]
    return (str(device),) + tuple((t.data_ptr(), t._version) for t in ts)


def layer_for(attn, device) -> BifrostLayer:
    """The BifrostLayer of a converted HybridAttention, rebuilt when its parameters changed (in-place updates
    bump the tensors' version counters) or the device differs."""
    key = _layer_key(attn, device)
    cached = attn.__dict__.get("_b200_layer")
    if cached is None or cached[0] != key:
        cached = (key, BifrostLayer.from_module(attn, device=device))
        attn.__dict__["_b200_layer"] = cached
    return cached[1]


def _student(self, x, q, k, v, qr, kr, start: int, cache=None, memory: bool = True):
    """HybridAttention._student (hibrit.py:363-424) on the fused B200 layer."""
    _require_cuda(x, q, k, v, qr, kr)
    return layer_for(self, x.device).student(x, q, k, v, qr, kr, int(start), cache, memory)


def _mem_inputs(self, x, q, k, pos):
    """HybridAttention._mem_inputs (hibrit.py:327-334): returns qm, km, g, beta."""
    _require_cuda(x, q, k, pos)
    qm, km, g, beta, _ = layer_for(self, x.device).mem_inputs(x, q, k, pos=pos)
    return qm, km, g, beta


def _window(self, qr, ext_k, ext_v, ext_pos, sink_k, sink_v, pos):
    """HybridAttention._window (hibrit.py:336-361): sinks + last-W window softmax; returns o [B,t,H,D], lse [B,H,t].

    The reference passes explicit key positions (``ext_pos``: the ring in time order, -1 for empty slots, then
    the new tokens) and query positions ``pos``.  The kernels take key j at position kpos0 + j; the positions
    are checked against that form (empty slots may only stand where the position is below the sinks, which
    the window excludes anyway) and any other layout raises NotImplementedError."""
    _require_cuda(qr, ext_k, ext_v, ext_pos, sink_k, sink_v, pos)
    t, n_ext = qr.shape[2], ext_k.shape[2]
    p = pos.to(torch.int64)
    # the positions are device tensors: their first value and the layout check come back in one read
    ar = torch.arange(max(t, n_ext), device=p.device, dtype=torch.int64)
    q0 = p[:1] if t else torch.zeros(1, dtype=torch.int64, device=p.device)
    expect = q0 - (n_ext - t) + ar[:n_ext]
    bad = ((ext_pos.to(torch.int64) != expect) & (expect >= self.sinks)).any()
    if t:
        bad = bad | (p != q0 + ar[:t]).any()
    qpos0, bad = torch.stack((q0[0], bad.to(torch.int64))).tolist()
    kpos0 = qpos0 - (n_ext - t)
    if bad:
        raise NotImplementedError("heimdall_b200 window: key/query positions must be contiguous "
                                  "(ring in time order followed by the new tokens)")
    if sink_k is not None and sink_k.shape[2] == 0:
        sink_k = sink_v = None
    return F_.window_attention(qr, ext_k, ext_v, qpos0, kpos0, self.sinks, self.window, sink_k, sink_v)


def _teacher(self, qr, kr, v, cache):
    """HybridAttention._teacher (hibrit.py:275-290): full attention of a kept layer over its growing cache, with
    the retrieval branch of ``set_retrieval`` (hibrit.py:292-324) for single-token decode."""
    _require_cuda(qr, kr, v)
    return R_.teacher(qr, kr, v, cache, getattr(self, "retrieval", None))


def window_attention(a, qr, kr, v):
    """heimdall.motor.window_attention (motor.py:105-115): the window and sinks of a whole sequence from an empty
    ring (positions 0 .. t-1), the cache-free path of HybridAttention._student.  Returns o [B,t,H,D], lse [B,H,t].

    The reference prepends W empty ring rows (position -1) and calls ``_window``; here the keys are the
    sequence itself from position 0, which the kernels take directly (no host read of the positions, no
    concatenated copies)."""
    _require_cuda(qr, kr, v)
    t = qr.shape[2]
    n = min(a.sinks, t)
    vt = v.transpose(1, 2)
    sk = kr[:, :, :n] if n else None
    sv = vt[:, :, :n] if n else None
    return F_.window_attention(qr, kr, vt, 0, 0, a.sinks, a.window, sk, sv)


# ---------------------------------------------------------------------------------------------- install
def install(modules=None) -> None:
    """Patch the reference package's Bifrost-path functions and HybridAttention methods (idempotent).

    Only ``PATCHED_NAMES`` change; the linear-attention ops (``kernels.delta_rule``, ``delta_rule_step`` and
    their copies in ``hibrit``) keep the reference's implementation."""
    if _SAVED:
        return
    m = _modules(modules)
    hibrit, motor = m["hibrit"], m["motor"]
    try:
        _patch(motor, "delta_rule_gqa", delta_rule_gqa)
        _patch(motor, "window_attention", window_attention)
        cls = hibrit.HybridAttention
        _patch(cls, "_student", _student)
        _patch(cls, "_mem_inputs", _mem_inputs)
        _patch(cls, "_window", _window)
        _patch(cls, "_teacher", _teacher)
    except Exception:
        uninstall()
        raise


def uninstall() -> None:
    """Restore every attribute ``install`` replaced."""
    while _SAVED:
        owner, name, value = _SAVED.pop()
        setattr(owner, name, value)


def installed() -> bool:
    return bool(_SAVED)


def self_test(device, reference) -> float:
    """The reference's prepare() check on this package's delta rule: seeded data of the shape used at
    kernels.py:170-176 with head dim 256 (the kernels' head dim), relative error of o and the final state
    against ``reference`` (the host package's delta_rule_reference)."""
    gen = torch.Generator().manual_seed(0)
    b, t, h, d = 2, 150, 2, 256
    q = torch.nn.functional.normalize(torch.randn(b, t, h, d, generator=gen), dim=-1) * d ** -0.5
    k = torch.nn.functional.normalize(torch.randn(b, t, h, d, generator=gen), dim=-1)
    v = torch.randn(b, t, h, d, generator=gen)
    g = -torch.rand(b, t, h, generator=gen) * 0.2
    beta = torch.rand(b, t, h, generator=gen)
    s0 = torch.randn(b, h, d, d, generator=gen) * 0.1
    ref_o, ref_s = reference(q, k, v, g, beta, 64, s0)
    o, s = F_.delta_rule(*(z.to(device) for z in (q, k, v, g, beta)), 64, s0.to(device))
    return max(((o.float().cpu() - ref_o).norm() / ref_o.norm()).item(),
               ((s.float().cpu() - ref_s).norm() / ref_s.norm()).item())


def prepare(device: torch.device, backend: str = "b200", modules=None) -> str:
    """The ``kernels.prepare`` convention for this package: self-test against the host package's
    ``delta_rule_reference``, then install.  Raises when the device is not CUDA or the self-test fails."""
    device = torch.device(device)
    if device.type != "cuda":
        raise RuntimeError("heimdall_b200 needs a CUDA device (there is no CPU fallback)")
    m = _modules(modules)
    reference = getattr(m["kernels"], "delta_rule_reference", None)
    if reference is None:
        raise RuntimeError("the host package has no delta_rule_reference to self-test against")
    err = self_test(device, reference)
    if not err < SELF_TEST_TOL:
        raise RuntimeError(f"heimdall_b200 delta rule failed the self-test (relative error {err:.4f})")
    install(m)
    return f"heimdall_b200 (relative error {err:.5f})"

"""heimdall_b200: Heimdall's Bifrost converted-layer hot path on NVIDIA B200 (sm_100a).

Host code is Python/PyTorch (device memory, streams, torch.distributed); all arithmetic of the path
runs in hand-written CUDA kernels behind the C ABI in ``include/bifrost_b200.h``
(``heimdall_b200/lib/libbifrost_b200.so``, built with ``python -m heimdall_b200.build``).
There is no CPU fallback: every op raises on CPU tensors or when the library is missing.

Public API (mirrors of the reference ``heimdall`` package):
  delta_rule                         heimdall/kernels.py:94-129, 152-155
  delta_rule_gqa                     heimdall/motor.py:70-102
  delta_rule_step                    heimdall/kernels.py:132-138
  window_attention                   heimdall/hibrit.py:336-361 (the math of _window_fp32)
  BifrostLayer.student               heimdall/hibrit.py:363-424 (HybridAttention._student)
  BifrostLayer.mem_inputs            heimdall/hibrit.py:327-334
  BifrostLayer.student_host          _student for host (pinned) inputs, copies overlapped with the layer
  BifrostLayer.decode_step           _student with t == 1 at a position per sequence (serving batches)
  BifrostLayer.student_varlen        _student over packed variable-length sequences (one prefill each)
  BifrostAttention.forward           heimdall/hibrit.py:426-432 (HybridAttention.forward, converted layer:
                                     projections, fused prologue / epilogue around the core)
  sp.student_sp                      one layer prefill of a sequence split over GPUs (sequence parallelism)
  plugin.prepare / install           the kernels.prepare plug-in convention (heimdall/kernels.py:158-188)
"""
from .functional import delta_rule, delta_rule_gqa, delta_rule_step, delta_rule_step_gqa, window_attention  # noqa: F401
from .layer import BifrostLayer  # noqa: F401
from .attention import BifrostAttention  # noqa: F401

__all__ = ["delta_rule", "delta_rule_gqa", "delta_rule_step", "delta_rule_step_gqa", "window_attention",
           "BifrostLayer", "BifrostAttention"]

"""Device-side failure detection on the GPU, exercised without any fault.

Every wait of the kernels is bounded: a wait that runs out records (site, block, thread) in the device
error record, the kernel unwinds and returns, and ``bf_device_error`` reports it.  ``bf_selftest_wait_timeout``
runs that path on purpose (a wait on an mbarrier phase that nothing completes, with a 2 ms limit).  The test
checks the report, that the record is cleared by the read, and that the context is still usable: a decode
state step right after it matches the oracle.
"""
import time

import pytest
import torch
import torch.nn.functional as F

from oracle import bifrost_oracle as ob

pytestmark = pytest.mark.gpu

BF_ERR_TIMEOUT = 6
SELFTEST_SITE = 0xF1


def test_bounded_wait_times_out_reports_and_recovers():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda")
    import heimdall_b200 as hb
    from heimdall_b200 import _lib
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.device_error(stream)[0] == 0
    t0 = time.perf_counter()
    _lib.call("bf_selftest_wait_timeout", 2000, stream)
    word, bx, byz, tid = _lib.device_error(stream)
    elapsed = time.perf_counter() - t0
    assert word == (SELFTEST_SITE << 8) | BF_ERR_TIMEOUT
    assert bx == 0 and byz == 0 and tid % 32 == 0 and tid < 128
    assert elapsed < 2.0
    assert _lib.device_error(stream)[0] == 0          # the read cleared the record
    # the context is still usable
    g_ = torch.Generator().manual_seed(3)
    B, H, D = 2, 4, 256
    q = F.normalize(torch.randn(B, H, D, generator=g_), dim=-1) * D ** -0.5
    k = F.normalize(torch.randn(B, H, D, generator=g_), dim=-1)
    v = torch.randn(B, H, D, generator=g_)
    g, beta = -torch.rand(B, H, generator=g_), torch.rand(B, H, generator=g_)
    s0 = torch.randn(B, H, D, D, generator=g_) * 0.1
    o_ref, s_ref = ob.gdn_step(q, k, v, g, beta, s0, dtype=torch.float64)
    o, s = hb.delta_rule_step(*(z.to(dev) for z in (q, k, v, g, beta, s0)))
    torch.cuda.synchronize()
    assert ob.rel_l2(o.cpu(), o_ref) < 1e-5 and ob.rel_l2(s.cpu(), s_ref) < 1e-5

"""Failure handling of the sequence-parallel prefill (heimdall_b200.sp) on CPU gloo ranks, with faults made on
the host only: a rank that leaves before the all-gather of the state maps, and a rank that sends a corrupted
(non-finite) map.  In both cases the surviving ranks must end with an exception within the process group's
timeout instead of hanging, and a corrupted map must be reported by every rank.

The layer engine is the CPU oracle stand-in of tests/test_sp.py (``OracleLayer``); a subclass injects the
fault in ``prefill_sp_begin``, which runs after the halo exchange and before the all-gather."""
import datetime
import json
import multiprocessing
import os
import time

import torch
import torch.distributed as dist

import test_sp as base
from params import layer_params

PG_TIMEOUT_S = 5


class LeavingLayer(base.OracleLayer):
    """Rank 1 leaves (raises and exits) before the all-gather."""

    def __init__(self, p, rank):
        super().__init__(p)
        self.rank = rank

    def prefill_sp_begin(self, *a):
        if self.rank == 1:
            raise SystemExit(3)
        return super().prefill_sp_begin(*a)


class CorruptingLayer(base.OracleLayer):
    """Rank 0 hands a state map with NaNs to the all-gather."""

    def __init__(self, p, rank):
        super().__init__(p)
        self.rank = rank

    def prefill_sp_begin(self, *a):
        M, N, h = super().prefill_sp_begin(*a)
        if self.rank == 0:
            M = M.clone()
            M[..., 0, 0] = float("nan")
        return M, N, h


def _rank(rank, world, port, kind, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))
    from heimdall_b200 import sp
    sp.F_.apply_prefix = base.oracle_apply_prefix
    p = layer_params(base.H, base.G, base.D, base.DM, window=base.W, sinks=base.S, archival=1, seed=5)
    layer = (LeavingLayer if kind == "leave" else CorruptingLayer)(p, rank)
    x, q, k, v, qr, kr = base._inputs()
    sl = slice(rank * base.T, (rank + 1) * base.T)
    t0 = time.monotonic()
    rec = {"rank": rank, "raised": None}
    try:
        sp.student_sp(layer, x[:, sl], q[:, sl], k[:, sl], v[:, sl], qr[:, :, sl], kr[:, :, sl])
    except RuntimeError as e:
        rec["raised"] = type(e).__name__
        rec["msg"] = str(e)[:300]
    rec["seconds"] = time.monotonic() - t0
    with open(f"{out_path}.{rank}", "w") as f:
        json.dump(rec, f)
    # no further collective: the peer may be gone
    os._exit(0)


def _run(kind, tmp_path):
    ctx = multiprocessing.get_context("spawn")
    port = base._free_port()
    out = str(tmp_path / kind)
    procs = [ctx.Process(target=_rank, args=(r, 2, port, kind, out)) for r in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=PG_TIMEOUT_S * 12)
    alive = [pr for pr in procs if pr.is_alive()]
    for pr in alive:
        pr.kill()
    assert not alive, "a rank hung instead of failing within the process-group timeout"
    recs = {}
    for r in range(2):
        path = f"{out}.{r}"
        if os.path.exists(path):
            with open(path) as f:
                recs[r] = json.load(f)
    return procs, recs


def test_rank_leaving_before_all_gather_fails_the_others(tmp_path):
    procs, recs = _run("leave", tmp_path)
    assert procs[1].exitcode == 3          # the rank that left
    assert 0 in recs and recs[0]["raised"] == "RuntimeError", recs
    assert recs[0]["seconds"] < PG_TIMEOUT_S * 6


def test_corrupted_state_map_is_reported_by_every_rank(tmp_path):
    procs, recs = _run("corrupt", tmp_path)
    assert all(pr.exitcode == 0 for pr in procs)
    for r in range(2):
        assert recs[r]["raised"] == "RuntimeError", recs
        assert "segment(s) [0]" in recs[r]["msg"]


def test_finite_check_flags_only_bad_segments():
    from heimdall_b200 import sp
    M = torch.zeros(3, 1, 2, 4, 4)
    N = torch.zeros_like(M)
    N[2, 0, 1, 3, 3] = float("inf")
    flags = sp._maps_finite(M, N)
    try:
        sp._raise_if_corrupted((flags, None))
        raise AssertionError("no error raised")
    except RuntimeError as e:
        assert "segment(s) [2]" in str(e)
    sp._raise_if_corrupted((sp._maps_finite(M, torch.zeros_like(M)), None))

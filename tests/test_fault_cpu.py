"""Fault injection on the host among CPU gloo ranks (no device work at all).

* a rank raises mid-training -> it publishes the failure and the survivor
  stops before its next step with ``PeerFailure`` naming that rank;
* a rank exits without a word -> the survivor sees the stale heartbeat and
  stops with ``PeerFailure``;
* a rank stalls -> its step watchdog ends it (exit 17), then as above;
* a collective with a vanished peer ends with an error at the process-group
  timeout instead of waiting forever;
* the step watchdog ends a stuck process with exit code 17.

The reference has no fault handling beyond its NCCL timeout
(``primus_dlrm/distributed/setup.py:30-31``).
"""
from __future__ import annotations

import os
import subprocess
import sys
import textwrap
import time
from pathlib import Path

import pytest

from tests.dist_utils import run_ranks_collect

ROOT = Path(__file__).resolve().parent.parent


def _trainer_rank(rank, world, mode):
    """Tiny DDP training; rank 1 misbehaves before its 4th batch."""
    import torch

    from primus_dlrm_b200.config import Config
    from primus_dlrm_b200.data.synthetic import generate_batch
    from primus_dlrm_b200.models.onetrans import OneTransModel
    from primus_dlrm_b200.parallel.health import PeerFailure
    from primus_dlrm_b200.parallel.wrapper import wrap_model
    from primus_dlrm_b200.training.engine import TrainEngine
    from primus_dlrm_b200.training.trainer import DistributedTrainer

    torch.set_num_threads(2)
    cfg = Config.load(ROOT / "configs" / "onetrans_tiny.yaml")
    cfg.data.history_length = 4
    cfg.train.batch_size = 8 * world
    cfg.train.kernels = "eager"
    cfg.train.heartbeat_timeout_s = 1.5
    if rank == 1 and mode == "stall":
        cfg.train.step_timeout_s = 3.0       # the stalled rank's own watchdog ends it (exit 17)
    cfg.distributed.embedding_sharding.enabled = False
    torch.manual_seed(0)
    model = OneTransModel(cfg)
    model, sync = wrap_model(model, torch.device("cpu"), cfg)
    eng = TrainEngine(model, cfg, torch.device("cpu"), grad_sync=sync, total_steps=20)
    batches = [generate_batch(cfg, 8, seed=rank * 100 + i) for i in range(8)]

    def loader():
        for i, b in enumerate(batches):
            if i == 3:
                if rank == 1:
                    if mode == "raise":
                        raise RuntimeError("injected failure")
                    if mode == "exit":
                        os._exit(3)
                    if mode == "stall":
                        time.sleep(30.0)
                else:
                    # let rank 1's failure (or silence) become visible first
                    time.sleep({"raise": 0.5, "exit": 2.5, "stall": 8.0}[mode])
            yield b

    tr = DistributedTrainer(model, eng, loader(), cfg, torch.device("cpu"), log_interval=100, run_dir="/tmp/_unused")
    try:
        tr.train()
    except PeerFailure as e:
        return {"peer_failure": e.rank, "reason": e.reason, "step": eng.global_step}
    return {"done": eng.global_step}


@pytest.mark.parametrize("mode", ["raise", "exit", "stall"])
def test_survivor_stops_between_steps(mode):
    t0 = time.monotonic()
    res, errs, codes = run_ranks_collect(_trainer_rank, 2, mode, timeout=120, pg_timeout=20)
    assert time.monotonic() - t0 < 100
    assert 0 in res, errs.get(0)
    r0 = res[0]
    assert r0.get("peer_failure") == 1, r0
    assert r0["step"] == 3, (r0, errs)        # stopped before launching step 4
    if mode == "raise":
        assert "injected failure" in r0["reason"]
        assert "injected failure" in errs[1]
    else:
        assert "no heartbeat" in r0["reason"]
    if mode == "exit":
        assert codes[1] == 3
    if mode == "stall":
        assert codes[1] == 17


def _collective_with_dead_peer(rank, world):
    import torch
    import torch.distributed as dist
    t = torch.ones(4)
    dist.all_reduce(t)                        # both ranks alive
    if rank == 1:
        os._exit(5)
    t0 = time.monotonic()
    try:
        dist.all_reduce(t)
    except Exception as e:  # noqa: BLE001
        return {"error": type(e).__name__, "waited": time.monotonic() - t0}
    return {"error": None}


def test_collective_with_dead_peer_times_out():
    res, errs, codes = run_ranks_collect(_collective_with_dead_peer, 2, timeout=90, pg_timeout=4)
    assert codes[1] == 5
    assert res[0]["error"] is not None, res
    assert res[0]["waited"] < 60


def test_watchdog_exits_stuck_process():
    code = textwrap.dedent(f"""
        import sys, time
        sys.path.insert(0, {str(ROOT)!r})
        from primus_dlrm_b200.training.trainer import Watchdog
        w = Watchdog(0.5)
        w.kick()
        time.sleep(30)
    """)
    t0 = time.monotonic()
    p = subprocess.run([sys.executable, "-c", code], timeout=60, capture_output=True, text=True)
    assert p.returncode == 17, p.stderr
    assert time.monotonic() - t0 < 30


def test_health_monitor_single_process_is_inert():
    from primus_dlrm_b200.parallel.health import HealthMonitor
    h = HealthMonitor(1.0)
    assert not h.enabled
    h.beat(3)
    h.check()
    h.report_failure("x")


@pytest.mark.parametrize("mode", ["raise", "exit"])
def test_every_survivor_of_three_stops(mode):
    """With three ranks, both survivors stop before the same step and name
    rank 1 as the origin: directly, or through the other survivor's report
    when that one published first (its reason carries rank 1's)."""
    res, errs, codes = run_ranks_collect(_trainer_rank, 3, mode, timeout=120, pg_timeout=20)
    for r in (0, 2):
        assert r in res, errs.get(r)
        assert res[r].get("peer_failure") in (1, 2 - r), res[r]
        assert res[r]["peer_failure"] == 1 or "rank 1" in res[r]["reason"], res[r]
        assert res[r]["step"] == 3, (res[r], errs)
    if mode == "exit":
        assert codes[1] == 3

"""Host-side peer health: heartbeats and failure notices in the c10d store.

The reference relies on a 30-minute NCCL timeout and Slurm's
``--kill-on-bad-exit`` (``primus_dlrm/distributed/setup.py:30-31``,
``scripts/launch_slurm.sh:138``): a dead rank leaves the others blocked in
their next collective until the timeout.  Here every rank publishes, in the
process group's key-value store,

* ``hb/<rank>`` -- ``"<last finished step> <unix time>"``, refreshed by a
  daemon thread every ``timeout_s / 4`` (liveness, not progress: a rank that
  is slow, evaluating or blocked in a collective keeps beating), and
* ``fail/<rank>`` -- the reason, when the rank raises (``report_failure``),

and before launching a step a rank calls ``check()``, which raises
``PeerFailure`` naming the rank when a peer reported a failure or its
heartbeat is older than ``timeout_s`` (the process is gone).  A rank that is
alive but stuck is ended by its own step watchdog (``trainer.Watchdog``),
after which its heartbeat stops too.  So the survivors stop between steps --
with none of their kernels or collectives in flight -- instead of entering a
collective that can never complete.  All of it is host code.  Heartbeat ages
compare wall clocks of different processes, so hosts of one job need
synchronised clocks (NTP) well within ``timeout_s``.
"""
from __future__ import annotations

import threading
import time

import torch.distributed as dist

_PREFIX = "primus_dlrm_b200/health"


class PeerFailure(RuntimeError):
    def __init__(self, rank: int, reason: str):
        super().__init__(f"peer rank {rank} failed: {reason}")
        self.rank = rank
        self.reason = reason


class HealthMonitor:
    """Heartbeat publisher + peer checker over the default group's store."""

    def __init__(self, timeout_s: float, store=None, rank: int | None = None, world: int | None = None,
                 check_interval: int = 1):
        self.timeout_s = float(timeout_s)
        self.enabled = self.timeout_s > 0 and dist.is_initialized() and dist.get_world_size() > 1
        self.rank = dist.get_rank() if rank is None and dist.is_initialized() else (rank or 0)
        self.world = dist.get_world_size() if world is None and dist.is_initialized() else (world or 1)
        self.check_interval = max(int(check_interval), 1)
        self._n = 0
        self._step = -1
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self.store = None
        if self.enabled:
            base = store if store is not None else dist.distributed_c10d._get_default_store()
            self.store = dist.PrefixStore(_PREFIX, base)
            self._publish()
            self._thread = threading.Thread(target=self._run, daemon=True, name="pd-heartbeat")
            self._thread.start()

    def _publish(self) -> None:
        with self._lock:
            self.store.set(f"hb/{self.rank}", f"{self._step} {time.time():.3f}")

    def _run(self) -> None:
        period = max(self.timeout_s / 4, 0.05)
        while not self._stop.wait(period):
            try:
                self._publish()
            except Exception:  # noqa: BLE001 -- the store went away with rank 0; check() reports it
                return

    def beat(self, step: int) -> None:
        """Record the last finished step (reported in failure messages)."""
        self._step = int(step)

    def stop(self) -> None:
        self._stop.set()

    def report_failure(self, reason: str) -> None:
        """Publish this rank's failure (best effort; never raises)."""
        if self.store is None:
            return
        self._stop.set()
        try:
            with self._lock:
                self.store.set(f"fail/{self.rank}", reason[:500])
        except Exception:  # noqa: BLE001 -- the store may be gone with rank 0
            pass

    def check(self) -> None:
        """Raise ``PeerFailure`` if a peer reported a failure or went silent."""
        if self.store is None:
            return
        self._n += 1
        if self._n % self.check_interval:
            return
        peers = [r for r in range(self.world) if r != self.rank]
        fails = [f"fail/{r}" for r in peers]
        # check() waits for missing keys: test existence first, per key
        with self._lock:
            for r, key in zip(peers, fails):
                if self.store.check([key]):
                    raise PeerFailure(r, self.store.get(key).decode())
            keys = [f"hb/{r}" for r in peers]
            present = [k for k in keys if self.store.check([k])]
            vals = self.store.multi_get(present) if present else []
        now = time.time()
        seen = dict(zip(present, vals))
        for r, k in zip(peers, keys):
            if k not in seen:
                continue
            step, t = seen[k].decode().split()
            if now - float(t) > self.timeout_s:
                raise PeerFailure(r, f"no heartbeat for {now - float(t):.1f} s (last step {step})")

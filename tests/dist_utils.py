"""Spawn helpers for multi-process CPU (gloo) tests."""
from __future__ import annotations

import os
import socket
import traceback

import torch.multiprocessing as mp


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world, port, fn, args, q, env, pg_timeout=60.0):
    import torch.distributed as dist
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    os.environ.update(env or {})
    try:
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=pg_timeout))
        out = fn(rank, world, *args)
        import io

        import torch
        buf = io.BytesIO()
        torch.save(out, buf)  # tensors by value: the child may exit before the parent reads
        q.put((rank, "ok", buf.getvalue()))
    except BaseException:  # report to the parent instead of hanging it
        q.put((rank, "err", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run_ranks(fn, world: int, *args, env: dict | None = None, timeout: float = 300.0) -> dict[int, object]:
    """Run ``fn(rank, world, *args)`` in ``world`` gloo processes; returns {rank: result}.
    Raises with the child's traceback if any rank failed."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, args, q, env)) for r in range(world)]
    for p in procs:
        p.start()
    results, errors = {}, []
    for _ in range(world):
        rank, status, val = q.get(timeout=timeout)
        if status == "ok":
            import io

            import torch
            results[rank] = torch.load(io.BytesIO(val), weights_only=False)
        else:
            errors.append(f"rank {rank}:\n{val}")
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    if errors:
        raise RuntimeError("\n".join(errors))
    return results


def run_ranks_collect(fn, world: int, *args, timeout: float = 120.0, pg_timeout: float = 60.0,
                      env: dict | None = None) -> tuple[dict[int, object], dict[int, str], dict[int, int]]:
    """Like ``run_ranks`` but tolerant of ranks that fail or vanish: returns
    ({rank: result}, {rank: traceback}, {rank: exit code}).  A rank that exits
    without reporting simply has no entry in the first two dicts."""
    import queue as _queue
    import time as _time
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, args, q, env, pg_timeout)) for r in range(world)]
    for p in procs:
        p.start()
    results, errors = {}, {}
    deadline = _time.monotonic() + timeout
    while len(results) + len(errors) < world and _time.monotonic() < deadline:
        try:
            rank, status, val = q.get(timeout=0.5)
        except _queue.Empty:
            if all(not p.is_alive() for p in procs) and q.empty():
                break
            continue
        if status == "ok":
            import io

            import torch
            results[rank] = torch.load(io.BytesIO(val), weights_only=False)
        else:
            errors[rank] = val
    codes = {}
    for r, p in enumerate(procs):
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
            p.join()
        codes[r] = p.exitcode
    return results, errors, codes

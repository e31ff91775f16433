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


def _entry(rank, world, port, fn, args, q, env):
    import torch.distributed as dist
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    os.environ.update(env or {})
    try:
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
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

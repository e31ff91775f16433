#!/usr/bin/env python3
"""Run a few training steps of a config at a chosen per-GPU batch, for kernel
profilers: every hot kernel of the step launches, on a case small enough for
``ncu --set full`` replays (a few GB on the device).

    python scripts/profile_step.py --batch 256 --steps 3
    ncu --set full --clock-control none -k regex:gemm_kernel -s 20 -c 1 -o prof \\
        python scripts/profile_step.py --batch 256 --steps 3

With ``--breakdown`` the device time of every kernel (torch.profiler, CUDA
activity) is printed per step, largest first.  With ``--copies`` the ATen ops
that launch copy / cast / concatenation kernels are listed with their device
time, shapes and the package source lines that called them.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--config", default=str(ROOT / "configs" / "bench_onetrans_v6_b200.yaml"))
    p.add_argument("--batch", type=int, default=256)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=2)
    p.add_argument("--breakdown", action="store_true")
    p.add_argument("--copies", action="store_true")
    p.add_argument("--trace", default="", help="write a Chrome trace (CPU + CUDA) of the steps to this path "
                                                  "(rank 0; run under torchrun for several ranks)")
    a = p.parse_args(argv)
    from primus_dlrm_b200.config import Config
    from primus_dlrm_b200.data.batch import PackedBatch
    from primus_dlrm_b200.data.synthetic import generate_batch
    from primus_dlrm_b200.parallel.build import build_training
    from primus_dlrm_b200.parallel.setup import get_rank, get_world_size, init_distributed
    cfg = Config.load(a.config)
    init_distributed(timeout_s=300)
    world, rank = get_world_size(), get_rank()
    cfg.train.batch_size = a.batch * world
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    model, eng = build_training(cfg, dev)
    b = PackedBatch(generate_batch(cfg, a.batch, seed=1 + rank)).to_device(dev)
    for _ in range(a.warmup):
        eng.step(b)
    torch.cuda.synchronize()
    if a.copies:
        return _copies(eng, b, a.steps)
    if a.trace:
        return _trace(eng, b, a.steps, a.trace, rank)
    if not a.breakdown:
        for _ in range(a.steps):
            eng.step(b)
        torch.cuda.synchronize()
        print(f"ok: {a.steps} steps, batch {a.batch}, peak {torch.cuda.max_memory_allocated() / 1e9:.1f} GB")
        return
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(a.steps):
            eng.step(b)
        torch.cuda.synchronize()
    rows = sorted(((k.device_time_total, k.count, k.key) for k in prof.key_averages() if k.device_time_total > 0),
                  reverse=True)
    tot = sum(r[0] for r in rows) or 1.0
    print(f"device time per step: {tot / a.steps / 1000:.3f} ms (batch {a.batch})")
    for t, c, k in rows[:40]:
        print(f"{t / a.steps / 1000:9.3f} ms/step {100 * t / tot:5.1f}%  n={c // a.steps:4d}  {k[:100]}")


def _trace(eng, b, steps: int, path: str, rank: int) -> None:
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            eng.step(b)
        torch.cuda.synchronize()
    if rank == 0:
        prof.export_chrome_trace(path)
        from primus_dlrm_b200.training.trace_analysis import idle_gaps, load_trace
        import json
        print(json.dumps(idle_gaps(load_trace(path), 50.0, 25), indent=1))


_COPY_OPS = ("aten::copy_", "aten::cat", "aten::clone", "aten::contiguous", "aten::to", "aten::_to_copy",
             "aten::index", "aten::fill_", "aten::zero_", "aten::zeros", "aten::zeros_like", "aten::add",
             "aten::mul", "aten::stack", "aten::pad", "aten::constant_pad_nd", "aten::sum", "aten::where")


def _copies(eng, b, steps: int) -> None:
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA], record_shapes=True,
                 with_stack=True) as prof:
        for _ in range(steps):
            eng.step(b)
        torch.cuda.synchronize()
    pkg = str(ROOT / "primus_dlrm_b200")
    agg: dict[tuple, list] = {}
    for ev in prof.events():
        if ev.name not in _COPY_OPS or ev.device_time_total <= 0:
            continue
        # innermost package frames only: the op's own caller inside the framework
        frames = [f for f in (ev.stack or []) if f.startswith(pkg)][:2]
        key = (ev.name, str(ev.input_shapes)[:90], " <- ".join(f[len(pkg) + 1:] for f in frames))
        slot = agg.setdefault(key, [0, 0.0])
        slot[0] += 1
        slot[1] += ev.device_time_total
    rows = sorted(agg.items(), key=lambda kv: -kv[1][1])
    tot = sum(v[1] for _, v in rows) or 1.0
    print(f"copy-like ATen ops: {tot / steps / 1000:.3f} ms/step device time")
    for (name, shapes, where), (n, t) in rows[:40]:
        print(f"{t / steps / 1000:8.3f} ms/step n={n // steps:3d} {name:18s} {shapes} @ {where}")


if __name__ == "__main__":
    main()

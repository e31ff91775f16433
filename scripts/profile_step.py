#!/usr/bin/env python3
"""Run a few training steps of a config at a chosen per-GPU batch, for kernel
profilers: every hot kernel of the step launches, on a case small enough for
``ncu --set full`` replays (a few GB on the device).

    python scripts/profile_step.py --batch 256 --steps 3
    ncu --set full --clock-control none -k regex:gemm_kernel -s 20 -c 1 -o prof \\
        python scripts/profile_step.py --batch 256 --steps 3

With ``--breakdown`` the device time of every kernel (torch.profiler, CUDA
activity) is printed per step, largest first.
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
    a = p.parse_args(argv)
    from primus_dlrm_b200.config import Config
    from primus_dlrm_b200.data.batch import PackedBatch
    from primus_dlrm_b200.data.synthetic import generate_batch
    from primus_dlrm_b200.parallel.build import build_training
    cfg = Config.load(a.config)
    cfg.train.batch_size = a.batch
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    model, eng = build_training(cfg, dev)
    b = PackedBatch(generate_batch(cfg, a.batch, seed=1)).to_device(dev)
    for _ in range(a.warmup):
        eng.step(b)
    torch.cuda.synchronize()
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


if __name__ == "__main__":
    main()

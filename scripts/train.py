#!/usr/bin/env python3
"""Single-GPU (or CPU) training entry point (reference ``scripts/train.py``):
the distributed trainer with a world of one, no torchrun needed."""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main(argv=None):
    p = argparse.ArgumentParser(description="Single-device training")
    p.add_argument("--config", default="configs/dlrm_baseline.yaml")
    p.add_argument("--processed-dir", default="data/processed", help="<data_root>/processed[_<size>]")
    p.add_argument("--device", default="cuda:0")
    p.add_argument("--max-steps", type=int, default=0)
    p.add_argument("--results-dir", default="results")
    p.add_argument("--run-name", default="train")
    p.add_argument("--log-interval", type=int, default=100)
    p.add_argument("--skip-eval", action="store_true")
    a = p.parse_args(argv)
    for k in ("RANK", "WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT"):
        os.environ.pop(k, None)
    if a.device.startswith("cuda:"):
        os.environ["LOCAL_RANK"] = a.device.split(":", 1)[1]
    spec = importlib.util.spec_from_file_location("_run_distributed", HERE / "run_distributed.py")
    rd = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(rd)
    args = ["--config", a.config, "--data-root", str(Path(a.processed_dir).parent), "--max-steps", str(a.max_steps),
            "--results-dir", a.results_dir, "--run-name", a.run_name, "--log-interval", str(a.log_interval)]
    if a.skip_eval:
        args.append("--skip-eval")
    return rd.main(args)


if __name__ == "__main__":
    main()

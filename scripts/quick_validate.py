#!/usr/bin/env python3
"""Quick end-to-end validation (reference ``scripts/quick_validate.py``): train
a few thousand steps on one device, then a global ranking eval over the
top-K popular items."""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main(argv=None):
    p = argparse.ArgumentParser(description="Short training run + eval")
    p.add_argument("--config", default="configs/dlrm_baseline.yaml")
    p.add_argument("--processed-dir", default="data/processed")
    p.add_argument("--device", default="cuda:0")
    p.add_argument("--max-steps", type=int, default=5000)
    p.add_argument("--log-interval", type=int, default=500)
    p.add_argument("--eval-top-k", type=int, default=5000, help="candidates = the K most popular items")
    p.add_argument("--results-dir", default="results")
    a = p.parse_args(argv)
    for k in ("RANK", "WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT"):
        os.environ.pop(k, None)
    if a.device.startswith("cuda:"):
        os.environ["LOCAL_RANK"] = a.device.split(":", 1)[1]
    spec = importlib.util.spec_from_file_location("_run_distributed", HERE / "run_distributed.py")
    rd = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(rd)
    return rd.main(["--config", a.config, "--data-root", str(Path(a.processed_dir).parent), "--max-steps",
                    str(a.max_steps), "--log-interval", str(a.log_interval), "--results-dir", a.results_dir,
                    "--run-name", "quick_validate", "--eval-num-candidates", str(a.eval_top_k)])


if __name__ == "__main__":
    main()

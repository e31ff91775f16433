#!/usr/bin/env python3
"""Evaluate a checkpoint for one task (reference ``scripts/evaluate.py``):
global ranking over the 5000 most popular items plus per-user ranking."""
from __future__ import annotations

import argparse
import importlib.util
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main(argv=None):
    p = argparse.ArgumentParser(description="Checkpoint evaluation for one task")
    p.add_argument("--config", default="configs/dlrm_baseline.yaml")
    p.add_argument("--checkpoint", required=True)
    p.add_argument("--processed-dir", default="data/processed")
    p.add_argument("--device", default="cuda:0")
    p.add_argument("--task", default="listen_plus", choices=["listen_plus", "like"])
    a = p.parse_args(argv)
    spec = importlib.util.spec_from_file_location("_eval_full", HERE / "eval_full.py")
    ef = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ef)
    common = ["--config", a.config, "--checkpoint", a.checkpoint, "--processed-dir", a.processed_dir,
              "--device", a.device, "--task", a.task]
    return (ef.main(common + ["--mode", "global", "--eval-top-k", "5000"]),
            ef.main(common + ["--mode", "peruser"]))


if __name__ == "__main__":
    main()

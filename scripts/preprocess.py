#!/usr/bin/env python3
"""Yambda preprocessing CLI (same flags as the reference's ``scripts/preprocess.py``):
raw ``multi_event.parquet`` -> GTS split, sessions, session index, item
popularity and split metadata under ``data/processed[_<size>]``."""
from __future__ import annotations

import argparse
import logging
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from primus_dlrm_b200.data.preprocessing import preprocess  # noqa: E402


def main(argv=None) -> Path:
    p = argparse.ArgumentParser(description="Preprocess the Yambda dataset")
    p.add_argument("--raw-dir", default="data/raw", help="raw data directory (holds <size>/multi_event.parquet)")
    p.add_argument("--out-dir", default=None, help="default: data/processed (50m) or data/processed_<size>")
    p.add_argument("--size", default="50m", choices=["50m", "500m", "5b"])
    p.add_argument("--session-gap", type=int, default=1800, help="session gap in seconds")
    p.add_argument("--train-days", type=int, default=300)
    p.add_argument("--gap-minutes", type=int, default=30)
    p.add_argument("--test-days", type=int, default=1)
    p.add_argument("--no-chunked", action="store_true", help="accepted for compatibility; reads are always by row group")
    a = p.parse_args(argv)
    logging.basicConfig(level=logging.INFO, format="%(asctime)s %(levelname)s %(message)s")
    raw = Path(a.raw_dir)
    out = Path(a.out_dir) if a.out_dir else raw.parent / ("processed" if a.size == "50m" else f"processed_{a.size}")
    return preprocess(raw, out, a.size, session_gap_seconds=a.session_gap, train_days=a.train_days,
                      gap_minutes=a.gap_minutes, test_days=a.test_days)


if __name__ == "__main__":
    main()

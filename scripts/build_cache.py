#!/usr/bin/env python3
"""Pre-build the flat event-store caches (reference ``scripts/build_cache.py``):
one cache per distinct (dataset size, counters, windows) variant, for the
train and/or eval split, so training jobs only map the ``.npy`` files."""
from __future__ import annotations

import argparse
import logging
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from primus_dlrm_b200.config import Config  # noqa: E402

logger = logging.getLogger("build_cache")


def _variants(args) -> list[Config]:
    if args.all_configs:
        seen, out = set(), []
        for f in sorted(Path(args.config_dir).glob("*.yaml")):
            try:
                c = Config.load(f)
            except Exception as e:  # noqa: BLE001 -- a broken config is skipped with a note
                logger.warning("skip %s: %s", f, e)
                continue
            if c.data.synthetic.enabled:
                continue
            key = (c.data.dataset_size, c.data.enable_counters, tuple(c.data.counter_windows_days),
                   c.data.history_length, tuple(sorted(c.data.history_lengths.items())))
            if key not in seen:
                seen.add(key)
                out.append(c)
        return out
    c = Config.load(args.config) if args.config else Config()
    if args.enable_counters:
        c.data.enable_counters = True
    if args.counter_windows:
        c.data.counter_windows_days = list(args.counter_windows)
    return [c]


def main(argv=None) -> list[str]:
    p = argparse.ArgumentParser(description="Pre-build the flat event-store caches")
    src = p.add_mutually_exclusive_group()
    src.add_argument("--config", default=None, help="one YAML config (its data section)")
    src.add_argument("--all-configs", action="store_true", help="every distinct variant under --config-dir")
    p.add_argument("--config-dir", default="configs")
    p.add_argument("--data-root", default=None, help="root of raw/processed/cache (default: config data_dir)")
    p.add_argument("--dataset-size", default=None, choices=["50m", "500m", "5b"])
    p.add_argument("--enable-counters", action="store_true")
    p.add_argument("--counter-windows", type=int, nargs="+", default=None)
    p.add_argument("--splits", nargs="+", default=["train", "eval"], choices=["train", "eval"])
    a = p.parse_args(argv)
    logging.basicConfig(level=logging.INFO, format="%(asctime)s %(levelname)s %(message)s")
    from primus_dlrm_b200.data.dataset import DataPaths, YambdaEvalDataset, YambdaTrainDataset
    built = []
    for cfg in _variants(a):
        if a.dataset_size:
            cfg.data.dataset_size = a.dataset_size
        cfg.data.use_cache = True
        paths = DataPaths.from_config(cfg.data, a.data_root)
        for split in a.splits:
            ds = (YambdaTrainDataset if split == "train" else YambdaEvalDataset)(cfg, paths)
            logger.info("%s cache ready: %d samples (%s, counters=%s)", split, len(ds), paths.cache,
                        cfg.data.enable_counters)
            built.append(f"{split}:{paths.cache}")
    return built


if __name__ == "__main__":
    main()

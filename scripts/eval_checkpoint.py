#!/usr/bin/env python3
"""Evaluate a checkpoint (``scripts/eval_checkpoint.py`` of the reference):
global top-N-popular candidates and per-user (train items, top-100) NDCG /
Recall@{10,50,100}.  Loads ``model_state_dict`` strictly into a plain model
(``_orig_mod.`` prefixes of compiled checkpoints are stripped).

    python scripts/eval_checkpoint.py --config C.yaml --checkpoint results/run/checkpoints/epoch_0.pt
"""
from __future__ import annotations

import argparse
import logging
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

logging.basicConfig(level=logging.INFO, format="%(asctime)s %(levelname)s %(message)s", stream=sys.stdout, force=True)
logger = logging.getLogger("eval_checkpoint")


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--config", required=True)
    p.add_argument("--checkpoint", required=True)
    p.add_argument("--processed-dir", default="data/processed",
                   help="<data_root>/processed[_<size>]; the data root is its parent")
    p.add_argument("--gpu", type=int, default=0)
    p.add_argument("--num-candidates", type=int, default=5000)
    p.add_argument("--log-interval", type=int, default=100)
    p.add_argument("--synthetic-users", type=int, default=0, help="evaluate on synthetic users instead")
    args = p.parse_args(argv)

    from primus_dlrm_b200.config import Config
    from primus_dlrm_b200.evaluation.metrics import evaluate_ranking, evaluate_ranking_peruser
    from primus_dlrm_b200.parallel.build import build_model
    from primus_dlrm_b200.training.checkpoint import load_checkpoint

    device = torch.device(f"cuda:{args.gpu}") if torch.cuda.is_available() else torch.device("cpu")
    config = Config.load(args.config)
    model = build_model(config, device=device)
    ckpt = load_checkpoint(args.checkpoint, model)
    model.eval()
    logger.info("Loaded checkpoint: step=%s, epoch=%s", ckpt.get("global_step"), ckpt.get("epoch"))
    task = config.task_names[0]
    if args.synthetic_users or config.data.synthetic.enabled:
        from primus_dlrm_b200.data.dataset import SyntheticEvalDataset
        ds = SyntheticEvalDataset(config, num_users=args.synthetic_users or 32)
        cands = np.random.default_rng(0).choice(ds.num_items, min(args.num_candidates, ds.num_items), replace=False)
    else:
        from primus_dlrm_b200.data.dataset import DataPaths, YambdaEvalDataset
        proc = Path(args.processed_dir)
        size = "50m" if proc.name == "processed" else proc.name.split("_", 1)[1]
        config.data.dataset_size = size
        ds = YambdaEvalDataset(config, DataPaths(proc.parent, size))
        cands = np.argsort(-ds.item_popularity)[: args.num_candidates]
    logger.info("Eval: %d users, %d candidates", len(ds), len(cands))
    t0 = time.time()
    rg = evaluate_ranking(model, ds, device, candidate_item_ids=cands, ks=[10, 50, 100], task=task,
                          log_interval=args.log_interval)
    logger.info("Global eval done in %.1fs", time.time() - t0)
    t0 = time.time()
    rp = evaluate_ranking_peruser(model, ds, device, ks=[10, 50, 100], task=task, top_n=100,
                                  log_interval=args.log_interval)
    logger.info("Per-user eval done in %.1fs", time.time() - t0)
    fmt = lambda d: " | ".join(f"{k}={v:.4f}" if isinstance(v, float) else f"{k}={v}" for k, v in sorted(d.items()))
    logger.info(f"[global-{args.num_candidates}] {fmt(rg)}")
    logger.info(f"[peruser-100] {fmt(rp)}")
    return rg, rp


if __name__ == "__main__":
    main()

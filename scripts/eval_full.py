#!/usr/bin/env python3
"""Ranking evaluation of a checkpoint (reference ``scripts/eval_full.py``):

* ``--mode global``  -- every test user against one candidate list: the full
  catalog (``--eval-top-k 0``) or the K most popular items;
* ``--mode peruser`` -- each user's own train items, metrics on the top-N;
* ``--mode mostpop`` -- the popularity baseline (no model).
"""
from __future__ import annotations

import argparse
import logging
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import numpy as np  # noqa: E402
import torch  # noqa: E402

logging.basicConfig(level=logging.INFO, format="%(asctime)s %(levelname)s %(message)s", stream=sys.stdout,
                    force=True)
logger = logging.getLogger("eval_full")


def main(argv=None) -> dict:
    p = argparse.ArgumentParser(description="Full ranking evaluation")
    p.add_argument("--config", required=True)
    p.add_argument("--processed-dir", default="data/processed")
    p.add_argument("--checkpoint", default=None)
    p.add_argument("--device", default="cuda:0" if torch.cuda.is_available() else "cpu")
    p.add_argument("--mode", choices=["global", "peruser", "mostpop"], default="global")
    p.add_argument("--task", default="listen_plus", choices=["listen_plus", "like"])
    p.add_argument("--eval-top-k", type=int, default=0, help="global mode: 0 = full catalog, K = top-K popular")
    p.add_argument("--top-n", type=int, default=100)
    p.add_argument("--score-batch-size", type=int, default=8192)
    a = p.parse_args(argv)
    from primus_dlrm_b200.config import Config
    from primus_dlrm_b200.data.dataset import DataPaths, YambdaEvalDataset
    from primus_dlrm_b200.evaluation.metrics import evaluate_ranking, evaluate_ranking_peruser
    from primus_dlrm_b200.evaluation.mostpop import mostpop_eval_dataset
    cfg = Config.load(a.config)
    proc = Path(a.processed_dir)
    size = "50m" if proc.name == "processed" else proc.name.split("_", 1)[1]
    cfg.data.dataset_size = size
    ds = YambdaEvalDataset(cfg, DataPaths(proc.parent, size))
    ks = [10, 50, 100]
    if a.mode == "mostpop":
        res = mostpop_eval_dataset(ds, a.task, ks, a.top_n)
    else:
        from primus_dlrm_b200.parallel.build import build_model
        from primus_dlrm_b200.training.checkpoint import load_checkpoint
        dev = torch.device(a.device)
        model = build_model(cfg, device=dev)
        if a.checkpoint:
            load_checkpoint(a.checkpoint, model)
        model.eval()
        with torch.no_grad():
            if a.mode == "global":
                cand = (np.arange(ds.num_items) if a.eval_top_k <= 0
                        else np.argsort(-ds.item_popularity)[: a.eval_top_k])
                res = evaluate_ranking(model, ds, dev, candidate_item_ids=cand, ks=ks, task=a.task,
                                       batch_size=a.score_batch_size)
            else:
                res = evaluate_ranking_peruser(model, ds, dev, ks=ks, task=a.task, top_n=a.top_n,
                                               batch_size=a.score_batch_size)
    logger.info("[%s %s] %s", a.mode, a.task, " | ".join(f"{k}={v:.4f}" if isinstance(v, float) else f"{k}={v}"
                                                         for k, v in sorted(res.items())))
    return res


if __name__ == "__main__":
    main()

#!/usr/bin/env python3
"""The Yambda paper's MostPop baseline on the raw event table (reference
``scripts/eval_mostpop.py``); expected on Yambda-50M listen+: NDCG@10 0.0186,
NDCG@100 0.0249, Recall@10 0.0064, Recall@100 0.0321."""
from __future__ import annotations

import argparse
import logging
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

logging.basicConfig(level=logging.INFO, format="%(asctime)s %(levelname)s %(message)s", stream=sys.stdout,
                    force=True)
logger = logging.getLogger("eval_mostpop")


def main(argv=None) -> dict:
    p = argparse.ArgumentParser(description="MostPop baseline (paper protocol)")
    p.add_argument("--data-file", default="data/raw/50m/multi_event.parquet")
    p.add_argument("--task", default="listen_plus", choices=["listen_plus", "like"])
    p.add_argument("--num-ranked", type=int, default=100)
    a = p.parse_args(argv)
    import pyarrow.parquet as pq

    from primus_dlrm_b200.evaluation.mostpop import mostpop_paper
    t = pq.read_table(a.data_file, columns=["uid", "item_id", "timestamp", "event_type", "played_ratio_pct"])
    col = lambda n: t.column(n).to_numpy(zero_copy_only=False)  # noqa: E731
    et = t.column("event_type")
    et = et.to_pylist() if "string" in str(et.type) or "dictionary" in str(et.type) else col("event_type")
    res = mostpop_paper(col("uid"), col("item_id"), col("timestamp"), et, col("played_ratio_pct"), a.task,
                        a.num_ranked)
    for k in (10, 50, 100):
        logger.info("  NDCG@%d = %.4f  |  Recall@%d = %.4f", k, res[f"ndcg@{k}"], k, res[f"recall@{k}"])
    logger.info("users evaluated: %d", res["num_users"])
    return res


if __name__ == "__main__":
    main()

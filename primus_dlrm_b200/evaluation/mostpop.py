"""MostPop baseline: one global popularity ranking for every user.

Two forms, as in the reference:
* ``mostpop_paper`` replicates the Yambda paper's protocol on the raw event
  table (``scripts/eval_mostpop.py``: last timestamp 26,000,000, a 1-day test
  window after a 30-minute gap, popularity = train events of the task);
* ``mostpop_eval_dataset`` ranks by listen+ counts of the training event
  store and scores a ``YambdaEvalDataset`` (``scripts/eval_full.py:193-222``).
Expected on Yambda-50M listen+: NDCG@10 0.0186, NDCG@100 0.0249,
Recall@10 0.0064, Recall@100 0.0321 (paper Table 6).
"""
from __future__ import annotations

import numpy as np

from primus_dlrm_b200.evaluation.metrics import metrics_from_ranking

LAST_TIMESTAMP = 26_000_000
DAY_SECONDS = 86_400
GAP_SECONDS = 30 * 60
TEST_SECONDS = DAY_SECONDS
LISTEN_THRESHOLD = 50


def _aggregate(per_user: list[dict], ks: list[int]) -> dict:
    out = {}
    for k in ks:
        for m in ("ndcg", "recall"):
            v = [u[f"{m}@{k}"] for u in per_user]
            out[f"{m}@{k}"] = float(np.mean(v)) if v else 0.0
    out["num_users"] = len(per_user)
    return out


def task_mask(event_type: np.ndarray, played_ratio: np.ndarray, task: str) -> np.ndarray:
    """Events that count for a task: listen+ (listen with >= 50 % played) or like."""
    et = np.asarray(event_type)
    if et.dtype.kind in "OUS":
        is_listen, is_like = et == "listen", et == "like"
    else:
        is_listen, is_like = et == 0, et == 1
    if task == "listen_plus":
        return is_listen & (np.nan_to_num(np.asarray(played_ratio, np.float64), nan=-1) >= LISTEN_THRESHOLD)
    if task == "like":
        return is_like
    raise ValueError(f"unknown task {task!r}")


def mostpop_paper(uid, item, ts, event_type, played_ratio, task: str = "listen_plus", num_ranked: int = 100,
                  ks=(10, 50, 100), last_timestamp: int = LAST_TIMESTAMP) -> dict:
    """The paper's split: train = [0, test_start - gap), test = [test_start, ...)."""
    m = task_mask(event_type, played_ratio, task)
    uid, item, ts = np.asarray(uid)[m], np.asarray(item)[m], np.asarray(ts)[m]
    test_start = last_timestamp - TEST_SECONDS
    tr = ts < test_start - GAP_SECONDS
    te = ts >= test_start
    counts = np.bincount(item[tr].astype(np.int64))
    # most popular first; ties broken by item id
    top = np.lexsort((np.arange(counts.size), -counts))[:num_ranked]
    te_uid, te_item = uid[te], item[te]
    keep = np.isin(te_uid, np.unique(uid[tr]))
    te_uid, te_item = te_uid[keep], te_item[keep]
    order = np.argsort(te_uid, kind="stable")
    te_uid, te_item = te_uid[order], te_item[order]
    bounds = np.flatnonzero(np.diff(te_uid)) + 1
    per_user = [metrics_from_ranking(top, set(grp.tolist()), list(ks))
                for grp in np.split(te_item, bounds) if grp.size]
    return _aggregate(per_user, list(ks))


def mostpop_eval_dataset(eval_dataset, task: str = "listen_plus", ks=(10, 50, 100), top_n: int = 100) -> dict:
    """Rank by listen+ counts of the training store; score every eval user."""
    st = eval_dataset.store
    ids = np.asarray(st.flat_item_ids)[np.asarray(st.flat_is_listen_plus, bool)]
    counts = np.bincount(ids.astype(np.int64), minlength=len(eval_dataset.item_popularity))
    top = np.argsort(-counts, kind="stable")[:top_n]
    per_user = []
    for idx in range(len(eval_dataset)):
        gt = eval_dataset[idx].get(f"ground_truth_{task}", set())
        if gt:
            per_user.append(metrics_from_ranking(top, gt, list(ks)))
    return _aggregate(per_user, list(ks))

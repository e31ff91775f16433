"""Ranking metrics and evaluation loops (``primus_dlrm/evaluation/metrics.py``).

``ndcg_at_k`` / ``recall_at_k`` take a ranked list of ``(item, score)`` (or a
dict item -> score) and a ground-truth set, exactly as in the reference.

Scoring differs from the reference (which runs one full forward per batch of
1024 candidates with the user's history tiled B times and sorts on the host):
``score_candidates`` batches candidates on the device and, for OneTrans,
uses the S-side cache: the causal mask makes the S tokens independent of the
NS (candidate) tokens, so S-token K/V are computed once per user and only the
NS tokens run per candidate (``OneTransModel.score_candidates``).  Top-k is
taken on the device.
"""
from __future__ import annotations

import logging
import math

import numpy as np
import torch

logger = logging.getLogger(__name__)


def _ranked(scores):
    if isinstance(scores, dict):
        return sorted(scores.items(), key=lambda x: x[1], reverse=True)
    return scores


def ndcg_at_k(scores, ground_truth: set[int], k: int) -> float:
    if len(ground_truth) == 0:
        return 0.0
    ranked = _ranked(scores)
    dcg = sum(1.0 / math.log2(i + 2) for i, (item, _) in enumerate(ranked[:k]) if item in ground_truth)
    idcg = sum(1.0 / math.log2(i + 2) for i in range(min(len(ground_truth), k)))
    return dcg / idcg if idcg > 0 else 0.0


def recall_at_k(scores, ground_truth: set[int], k: int) -> float:
    if len(ground_truth) == 0:
        return 0.0
    top = {item for item, _ in _ranked(scores)[:k]}
    return len(top & ground_truth) / len(ground_truth)


def metrics_from_ranking(ranked_items: np.ndarray, ground_truth: set[int], ks: list[int]) -> dict[str, float]:
    pairs = [(int(i), 0.0) for i in ranked_items]
    out = {}
    for k in ks:
        out[f"ndcg@{k}"] = ndcg_at_k(pairs, ground_truth, k)
        out[f"recall@{k}"] = recall_at_k(pairs, ground_truth, k)
    return out


def _aggregate(per_user: list[dict[str, float]], ks: list[int]) -> dict[str, float]:
    res: dict[str, float] = {}
    for k in ks:
        for m in ("ndcg", "recall"):
            vals = [u[f"{m}@{k}"] for u in per_user]
            res[f"{m}@{k}"] = float(np.mean(vals)) if vals else 0.0
    res["num_users"] = len(per_user)
    return res


@torch.no_grad()
def score_candidates(model, user_batch: dict[str, torch.Tensor], candidate_batch: dict[str, torch.Tensor],
                     task: str, batch_size: int = 1024) -> torch.Tensor:
    """Scores [C] of one user's history against C candidates (device tensor).

    ``user_batch`` holds the user-side tensors with a leading dim of 1;
    ``candidate_batch`` holds per-candidate tensors with leading dim C.
    """
    inner = getattr(model, "module", model)
    if hasattr(inner, "score_candidates"):
        from primus_dlrm_b200.parallel.fsdp import full_params
        with full_params(inner):          # FSDP units: the scorer reads block weights directly
            return inner.score_candidates(user_batch, candidate_batch, task, batch_size)
    C = next(iter(candidate_batch.values())).shape[0]
    out = []
    for s in range(0, C, batch_size):
        e = min(s + batch_size, C)
        b = {k: v[s:e] for k, v in candidate_batch.items()}
        for k, v in user_batch.items():
            b[k] = v.expand(e - s, *v.shape[1:])
        dev_type = next(iter(b.values())).device.type
        with torch.autocast(dev_type, dtype=torch.bfloat16, enabled=dev_type == "cuda"):
            out.append(model(b)[task].float())
    return torch.cat(out)


def evaluate_ranking(model, eval_dataset, device, candidate_item_ids=None, ks=None, task: str = "listen_plus",
                     batch_size: int = 1024, log_interval: int = 0) -> dict[str, float]:
    """Global candidate list (default: top popular items) per test user."""
    ks = ks or [10, 100]
    model.eval()
    if candidate_item_ids is None:
        candidate_item_ids = np.argsort(-eval_dataset.item_popularity)[:10000]
    cand = eval_dataset.candidate_batch(candidate_item_ids, device)
    per_user = []
    for idx in range(len(eval_dataset)):
        sample = eval_dataset[idx]
        gt = sample.get(f"ground_truth_{task}", set())
        if not gt:
            continue
        ub = eval_dataset.user_batch(sample, device)
        s = score_candidates(model, ub, eval_dataset.with_user_features(cand, sample, candidate_item_ids, device),
                             task, batch_size)
        order = torch.argsort(s, descending=True)[: max(ks)].cpu().numpy()
        per_user.append(metrics_from_ranking(np.asarray(candidate_item_ids)[order], gt, ks))
        if log_interval and (idx + 1) % log_interval == 0:
            logger.info("  [global] %d/%d users evaluated", idx + 1, len(eval_dataset))
    return _aggregate(per_user, ks)


def evaluate_ranking_peruser(model, eval_dataset, device, ks=None, task: str = "listen_plus", top_n: int = 100,
                             batch_size: int = 1024, log_interval: int = 0) -> dict[str, float]:
    """Per-user candidates = the user's unique train items; metrics on the top-N."""
    ks = ks or [10, 50, 100]
    model.eval()
    per_user = []
    for idx in range(len(eval_dataset)):
        sample = eval_dataset[idx]
        gt = sample.get(f"ground_truth_{task}", set())
        if not gt:
            continue
        items = eval_dataset.get_user_train_items(sample["uid"])
        if len(items) == 0:
            continue
        cand = eval_dataset.candidate_batch(items, device)
        ub = eval_dataset.user_batch(sample, device)
        s = score_candidates(model, ub, eval_dataset.with_user_features(cand, sample, items, device), task,
                             batch_size)
        order = torch.argsort(s, descending=True)[:top_n].cpu().numpy()
        per_user.append(metrics_from_ranking(np.asarray(items)[order], gt, ks))
        if log_interval and (idx + 1) % log_interval == 0:
            logger.info("  [peruser] %d/%d users evaluated", idx + 1, len(eval_dataset))
    return _aggregate(per_user, ks)

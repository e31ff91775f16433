"""Losses (``primus_dlrm/training/losses.py``).

``MultiTaskLoss``: weighted sum of per-task BCE-with-logits, or MSE for
``regression_tasks``.  ``InBatchBPRLoss``: in-batch BPR over a ``[B, B]``
user x item score matrix, averaged over positive anchors.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F


class MultiTaskLoss(nn.Module):
    def __init__(self, weights: dict[str, float] | None = None, regression_tasks: list[str] | None = None):
        super().__init__()
        weights = weights or {"task0": 1.0}
        self.weights = {k: v for k, v in weights.items() if v > 0}
        self._regression = set(regression_tasks or [])

    def forward(self, predictions: dict[str, torch.Tensor], labels: dict[str, torch.Tensor], **_):
        losses = {}
        for task in self.weights:
            if task not in predictions or task not in labels:
                continue
            p, y = predictions[task].float(), labels[task].float()
            losses[task] = F.mse_loss(p, y) if task in self._regression else \
                F.binary_cross_entropy_with_logits(p, y)
        total = sum(self.weights[k] * v for k, v in losses.items())
        return total, losses


class InBatchBPRLoss(nn.Module):
    """loss = mean over positive anchors i and negatives j != i of
    -log sigmoid((s_ii - s_ij) / T).  No host sync: anchors are masked."""

    def __init__(self, temperature: float = 0.1):
        super().__init__()
        self.temperature = temperature

    def forward(self, cross_scores: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        B = cross_scores.shape[0]
        s = cross_scores.float()
        pos = labels.bool()
        diag = s.diagonal()
        diff = (diag.unsqueeze(1) - s) / self.temperature
        eye = torch.eye(B, dtype=torch.bool, device=s.device)
        per = -F.logsigmoid(diff).masked_fill(eye, 0.0)
        per = per * pos.unsqueeze(1)
        n_pos = pos.sum()
        denom = (n_pos * (B - 1)).clamp_min(1).to(s.dtype)
        return per.sum() / denom

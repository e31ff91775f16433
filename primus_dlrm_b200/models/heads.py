"""Multi-task prediction heads (``primus_dlrm/models/heads.py:8-29``)."""
from __future__ import annotations

import torch
import torch.nn as nn

from primus_dlrm_b200.ops.loss import heads_loss


class MultiTaskHead(nn.Module):
    """``heads.<task>`` = Linear(D, 1) per task; ``forward`` -> {task: [B]}."""

    def __init__(self, input_dim: int, tasks: list[str] | None = None, device=None):
        super().__init__()
        self.tasks = list(tasks or ["task0"])
        self.heads = nn.ModuleDict({t: nn.Linear(input_dim, 1, device=device) for t in self.tasks})

    def forward(self, x: torch.Tensor) -> dict[str, torch.Tensor]:
        return {t: h(x).squeeze(-1) for t, h in self.heads.items()}


def fused_heads_loss(heads: nn.ModuleDict, h: torch.Tensor, batch: dict[str, torch.Tensor],
                     loss_weights: dict[str, float], regression_tasks: list[str]):
    """Heads + weighted multi-task loss in one fused op.

    Returns ``(total_loss, {task: loss}, {task: logits})``; tasks without a
    label in ``batch`` or with weight <= 0 are excluded from the loss.
    """
    tasks = [t for t in heads if loss_weights.get(t, 0) > 0 and t in batch]
    if not tasks:
        raise ValueError("no labelled task with a positive loss weight in the batch")
    W = torch.cat([heads[t].weight for t in tasks], dim=0)
    b = torch.cat([heads[t].bias for t in tasks], dim=0)
    labels = torch.stack([batch[t].float() for t in tasks], dim=0)
    if h.dtype != torch.bfloat16 and h.is_cuda:
        h = h.to(torch.bfloat16)
    total, per, logits = heads_loss(h, W, b, labels, [loss_weights[t] for t in tasks],
                                    [1 if t in regression_tasks else 0 for t in tasks])
    return total, {t: per[i] for i, t in enumerate(tasks)}, {t: logits[i] for i, t in enumerate(tasks)}

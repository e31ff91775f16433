"""Model interface (``primus_dlrm/models/base.py:10-40``).

``forward(batch) -> {task: logits [B]}``; ``forward_with_cross_scores``
adds the ``[B, B]`` user x item score matrix used by the in-batch BPR loss.
Models here additionally implement ``forward_loss(batch, loss_weights,
regression_tasks)`` which fuses the task heads with the multi-task loss.
"""
from __future__ import annotations

import torch
import torch.nn as nn


class BaseModel(nn.Module):
    def forward(self, batch: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:  # pragma: no cover
        raise NotImplementedError

    def forward_with_cross_scores(self, batch: dict[str, torch.Tensor], cross_task: str = ""):
        raise NotImplementedError

    def get_num_flops_per_sample(self) -> float:
        return 0.0

"""Assemble model + training engine for this rank.

world == 1: every table and parameter on the local device.
world  > 1: embedding tables sharded per the plan (row-wise / table-wise /
column-wise / data-parallel), dense parameters replicated with a flat
gradient all-reduce (DDP) or sharded (FSDP).
"""
from __future__ import annotations

import torch

from primus_dlrm_b200.config import Config
from primus_dlrm_b200.parallel.setup import get_world_size
from primus_dlrm_b200.training.engine import TrainEngine


def build_model(config: Config, device=None, meta_device: bool = False):
    """Model by ``config.model.model_type`` (``scripts/run_distributed.py:105-116``)."""
    from primus_dlrm_b200.models.dlrm import DLRMBaseline
    from primus_dlrm_b200.models.onetrans import OneTransModel
    mt = config.model.model_type
    if mt == "onetrans":
        return OneTransModel(config, device=device, meta_device=meta_device)
    if mt == "dlrm":
        return DLRMBaseline(config, device=device, meta_device=meta_device)
    raise ValueError(f"Invalid model type: {mt}")


def build_training(config: Config, device: torch.device, total_steps: int | None = None):
    """Returns (model, engine) ready to step on this rank."""
    world = get_world_size()
    if world <= 1:
        model = build_model(config, device=device)
        return model, TrainEngine(model, config, device, total_steps=total_steps)
    from primus_dlrm_b200.parallel.wrapper import wrap_model
    model = build_model(config, device=device, meta_device=True)
    model, grad_sync = wrap_model(model, device, config)
    return model, TrainEngine(model, config, device, grad_sync=grad_sync, total_steps=total_steps)

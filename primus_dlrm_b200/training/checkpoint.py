"""Checkpoints (``primus_dlrm/training/dist_trainer.py:723-756`` layout, plus resume).

File: ``torch.save({"epoch", "global_step", "model_state_dict", ...})`` at
``<run>/checkpoints/epoch_{epoch}.pt`` -- the reference's keys and weight
layout, so reference checkpoints load here and ours load in tools built for
the reference.  Additive optional keys enable resume (the reference saves
weights only): ``optimizer_state_dict`` (dense), ``sparse_optimizer_state``
({table: [state]}), ``scheduler_state_dict``, ``rng_state``, ``config``.

Sharded tables are gathered to rank 0 (``parallel.state.full_state_dict``).
Writes are atomic: a temporary file in the same directory, then rename.
"""
from __future__ import annotations

import logging
import os
from dataclasses import asdict
from pathlib import Path

import torch
import torch.distributed as dist

from primus_dlrm_b200.parallel.state import full_state_dict, load_full_state_dict, load_sparse_state

logger = logging.getLogger(__name__)


def _rank() -> int:
    return dist.get_rank() if dist.is_initialized() else 0


def save_checkpoint(path: str | Path, model, epoch: int, global_step: int, engine=None, config=None,
                    with_resume_state: bool = True) -> Path | None:
    """Collective when distributed (every rank must call it)."""
    path = Path(path)
    sd = full_state_dict(model, with_optimizer_state=with_resume_state)
    # gathered on every rank (collective when the optimizer state is sharded)
    opt_sd = engine.full_optimizer_state() if with_resume_state and engine is not None else None
    if _rank() != 0:
        return None
    sparse = sd.pop("__sparse_state__", None)
    payload = {"epoch": int(epoch), "global_step": int(global_step), "model_state_dict": sd}
    if with_resume_state:
        if engine is not None:
            payload["optimizer_state_dict"] = opt_sd
            payload["scheduler_state_dict"] = engine.scheduler.state_dict()
            sopt = getattr(engine, "sparse_opt", None)
            if sopt is not None:
                payload["sparse_optimizer_step"] = sopt.step
        if sparse is not None:
            payload["sparse_optimizer_state"] = sparse
        payload["rng_state"] = {"cpu": torch.get_rng_state(),
                                "cuda": torch.cuda.get_rng_state_all() if torch.cuda.is_available() else []}
        if config is not None:
            payload["config"] = asdict(config)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(f".{path.name}.tmp.{os.getpid()}")
    torch.save(payload, tmp)
    os.replace(tmp, path)
    logger.info("Saved checkpoint: %s", path)
    return path


def load_checkpoint(path: str | Path, model, engine=None, strict: bool = True) -> dict:
    """Load weights (and, if present and ``engine`` is given, the resume state).

    Raises ``RuntimeError`` with the file name for truncated or corrupted files.
    """
    path = Path(path)
    try:
        ckpt = torch.load(path, map_location="cpu", weights_only=False)
    except Exception as e:
        raise RuntimeError(f"cannot read checkpoint {path}: {type(e).__name__}: {e}") from e
    if not isinstance(ckpt, dict) or "model_state_dict" not in ckpt:
        raise RuntimeError(f"{path} is not a training checkpoint (no model_state_dict)")
    load_full_state_dict(model, ckpt["model_state_dict"], strict=strict)
    if "sparse_optimizer_state" in ckpt:
        load_sparse_state(model, ckpt["sparse_optimizer_state"])
    if engine is not None:
        if engine.flat is not None:
            engine.flat.rebind()
        if "optimizer_state_dict" in ckpt:
            engine.optimizer.load_state_dict(ckpt["optimizer_state_dict"])
        if "scheduler_state_dict" in ckpt:
            engine.scheduler.load_state_dict(ckpt["scheduler_state_dict"])
        engine.global_step = int(ckpt.get("global_step", 0))
        if getattr(engine, "sparse_opt", None) is not None and "sparse_optimizer_step" in ckpt:
            engine.sparse_opt.step = int(ckpt["sparse_optimizer_step"])
    if "rng_state" in ckpt:
        torch.set_rng_state(ckpt["rng_state"]["cpu"])
        # the CUDA generator of this process's device (dropout, on-device
        # sampling); only the current device is touched, so no other GPU gets
        # a context
        cuda_states = ckpt["rng_state"].get("cuda") or []
        if torch.cuda.is_available() and cuda_states:
            dev = torch.cuda.current_device()
            if dev < len(cuda_states):
                torch.cuda.set_rng_state(cuda_states[dev], device=dev)
    return ckpt


def latest_checkpoint(run_dir: str | Path) -> Path | None:
    d = Path(run_dir) / "checkpoints"
    cands = sorted(d.glob("epoch_*.pt"), key=lambda p: int(p.stem.split("_")[1]) if p.stem.split("_")[1].isdigit() else -1)
    return cands[-1] if cands else None

"""Distributed wrapping of a model (``primus_dlrm/distributed/wrapper.py:27-79``).

``wrap_model(model, device, config) -> (model, grad_sync)``:

* embedding tables are sharded by the plan (``parallel.planner``) whenever
  ``distributed.embedding_sharding.enabled`` or ``dense_strategy == "dmp"``;
  otherwise they are replicated (data-parallel with a sparse gradient
  all-gather), which is what the reference's plain DDP run does;
* dense parameters are broadcast from rank 0 and their gradients are
  synchronised by ``FlatGradSync`` (``ddp`` / ``dmp``: all-reduce of the flat
  gradient arena in buckets) or ``ShardedGradSync`` (``fsdp``:
  reduce-scatter of gradients, AdamW on this rank's 1/W slice, all-gather of
  parameters -- optimizer state and gradients sharded ZeRO-style).

``distributed.comm`` picks the sparse exchange: ``peer`` (NVLink peer-memory
kernels, CUDA) or ``nccl`` (collective baseline; also the CPU/gloo path).
"""
from __future__ import annotations

import logging

import torch
import torch.distributed as dist
import torch.nn as nn

from primus_dlrm_b200.parallel.planner import build_topology, log_plan, plan_tables
from primus_dlrm_b200.parallel.setup import get_rank, get_world_size
from primus_dlrm_b200.parallel.sharded_embedding import shard_embeddings

logger = logging.getLogger(__name__)


class FlatGradSync:
    """Average the flat dense-gradient arena over ranks (bucketed all-reduce)."""

    def __init__(self, group=None, bucket_mb: float = 256.0):
        self.group = group
        self.world = dist.get_world_size(group)
        self.bucket = int(bucket_mb * 2 ** 20 / 4)

    def sync(self, flat_grad: torch.Tensor) -> None:
        n = flat_grad.numel()
        works = []
        for s in range(0, n, self.bucket):
            works.append(dist.all_reduce(flat_grad[s:s + self.bucket], group=self.group, async_op=True))
        for w in works:
            w.wait()
        flat_grad.mul_(1.0 / self.world)


class ShardedGradSync:
    """ZeRO-style: reduce-scatter gradients so each rank owns 1/W of them,
    update that slice, all-gather the parameters (``fsdp`` strategy)."""

    sharded = True

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def shard_range(self, n: int) -> tuple[int, int]:
        per = -(-n // self.world)
        per = (per + 63) // 64 * 64
        a = min(self.rank * per, n)
        return a, min(a + per, n)

    def sync(self, flat_grad: torch.Tensor) -> None:
        n = flat_grad.numel()
        per = (-(-n // self.world) + 63) // 64 * 64
        pad = per * self.world - n
        g = torch.nn.functional.pad(flat_grad, (0, pad)) if pad else flat_grad
        out = torch.empty(per, dtype=g.dtype, device=g.device)
        dist.reduce_scatter_tensor(out, g, group=self.group)
        a, b = self.shard_range(n)
        flat_grad.zero_()
        flat_grad[a:b].copy_(out[: b - a]).mul_(1.0 / self.world)

    def gather_params(self, flat_data: torch.Tensor) -> None:
        n = flat_data.numel()
        per = (-(-n // self.world) + 63) // 64 * 64
        a, b = self.shard_range(n)
        mine = torch.zeros(per, dtype=flat_data.dtype, device=flat_data.device)
        mine[: b - a] = flat_data[a:b]
        full = torch.empty(per * self.world, dtype=flat_data.dtype, device=flat_data.device)
        dist.all_gather_into_tensor(full, mine, group=self.group)
        flat_data.copy_(full[:n])


def broadcast_dense(model: nn.Module, group=None) -> None:
    for p in model.parameters():
        if p.requires_grad:
            dist.broadcast(p.data, src=0, group=group)


def wrap_model(model: nn.Module, device: torch.device, config, group=None):
    world = get_world_size()
    rank = get_rank()
    dc = config.distributed
    if world <= 1:
        return model.to(device), None
    inner = getattr(model, "module", model)
    emb = getattr(inner, "emb", None)
    if emb is not None:
        comm = dc.comm if device.type == "cuda" else "nccl"
        if dc.embedding_sharding.enabled or dc.dense_strategy == "dmp":
            plans = plan_tables(config, world, build_topology(config, world))
        else:
            from primus_dlrm_b200.parallel.planner import TablePlan
            plans = {t.name: TablePlan(t.name, "data_parallel", ranks=list(range(world)), reason="ddp")
                     for t in emb.tables()}
        if rank == 0:
            log_plan(plans)
        shard_embeddings(emb, plans, rank, world, device, comm=comm, group=group,
                         seed=config.train.seed, init=config.model.embedding_init)
    model = model.to(device)
    broadcast_dense(model, group)
    if dc.dense_strategy == "fsdp":
        sync = ShardedGradSync(group)
    elif dc.dense_strategy in ("ddp", "dmp"):
        sync = FlatGradSync(group)
    else:
        raise ValueError(f"Unknown dense_strategy: {dc.dense_strategy!r}")
    logger.info("wrapped for %d ranks: dense=%s embeddings=%s comm=%s", world, dc.dense_strategy,
                "sharded" if emb is not None and emb.sharded else "none", dc.comm)
    return model, sync


def _has_meta_dense(model: nn.Module) -> bool:
    return any(p.device.type == "meta" and p.requires_grad for p in model.parameters())


def is_dmp(model: nn.Module) -> bool:
    inner = getattr(model, "module", model)
    emb = getattr(inner, "emb", None)
    return bool(emb is not None and getattr(emb, "sharded", False))

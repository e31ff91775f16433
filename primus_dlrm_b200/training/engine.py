"""One training step: forward (+fused heads/loss), backward (+fused sparse
optimizer), dense-gradient sync, clip + AdamW, LR schedules.

This is the step the reference runs in ``DistributedTrainer._sequential_steps``
(``primus_dlrm/training/dist_trainer.py:460-482``) with the following changes:

* dense parameters live in one flat fp32 arena; clip + AdamW are two fused
  launches and the data-parallel gradient sync works on slices of one buffer;
* bf16 autocast without a GradScaler (it is a no-op for bf16,
  ``dist_trainer.py:339-345``);
* the loss is not read back to the host inside ``step`` (the reference defers
  ``.item()`` to log steps too, ``dist_trainer.py:611-615``).
"""
from __future__ import annotations

import os

import math
import time

import torch
import torch.distributed as dist
import torch.nn as nn
from torch.optim.lr_scheduler import CosineAnnealingLR, LinearLR, SequentialLR

from primus_dlrm_b200.config import Config
from primus_dlrm_b200.data.batch import PackedBatch
from primus_dlrm_b200.ops.optim import FlatParams, FusedAdamW
from primus_dlrm_b200.training.losses import InBatchBPRLoss, MultiTaskLoss
from primus_dlrm_b200.utils.nvtx import phase


def dense_parameters(model: nn.Module) -> list[nn.Parameter]:
    """Trainable parameters that are not embedding tables (tables are updated
    by the fused sparse optimizer and have requires_grad=False)."""
    return [p for p in model.parameters() if p.requires_grad]


class TrainEngine:
    def __init__(self, model: nn.Module, config: Config, device: torch.device,
                 grad_sync=None, total_steps: int | None = None, dense_optimizer=None):
        self.model = model
        self.config = config
        self.device = torch.device(device)
        tc = config.train
        self.tasks = [k for k, v in tc.loss_weights.items() if v > 0]
        # fsdp: parameters are DTensor shards owned by FSDP; no flat arena
        self.fsdp = bool(getattr(grad_sync, "fsdp", False))
        self.flat = None if self.fsdp else FlatParams(dense_parameters(model))
        if dense_optimizer is not None:
            self.optimizer = dense_optimizer
        elif self.fsdp:
            if tc.dense_optimizer != "adamw":
                raise ValueError("dense_strategy 'fsdp' supports dense_optimizer 'adamw' only")
            from primus_dlrm_b200.parallel.fsdp import ShardedAdamW
            self.optimizer = ShardedAdamW(dense_parameters(model), lr=tc.lr, weight_decay=tc.weight_decay,
                                          max_grad_norm=tc.grad_clip, group=grad_sync.group)
        elif tc.dense_optimizer == "adamw":
            self.optimizer = FusedAdamW(self.flat, lr=tc.lr, weight_decay=tc.weight_decay,
                                        max_grad_norm=tc.grad_clip)
        elif tc.dense_optimizer == "shampoo":
            self.optimizer = _make_shampoo(self.flat.params, tc)
        else:
            raise ValueError(f"Unknown dense_optimizer='{tc.dense_optimizer}'. Supported: 'adamw', 'shampoo'")
        total = total_steps if total_steps is not None else max(tc.epochs, 1) * 10_000_000
        warm = LinearLR(self.optimizer, start_factor=tc.warmup_start_factor, total_iters=max(tc.warmup_steps, 1))
        cos = CosineAnnealingLR(self.optimizer, T_max=max(total - tc.warmup_steps, 1))
        self.scheduler = SequentialLR(self.optimizer, [warm, cos], milestones=[max(tc.warmup_steps, 1)])
        self.loss_fn = MultiTaskLoss(tc.loss_weights, tc.regression_tasks)
        self.bpr = InBatchBPRLoss(tc.contrastive_temperature) if tc.contrastive_weight > 0 else None
        self.grad_sync = grad_sync
        if grad_sync is not None and hasattr(grad_sync, "bind"):
            grad_sync.bind(self.flat)      # peer collectives: the arenas live in shared memory
        self.global_step = 0
        self.skipped_steps = 0
        self.use_amp = tc.bf16
        inner = getattr(model, "module", model)
        self.sparse_opt = inner.emb.optimizer if hasattr(inner, "emb") else None
        self._loss_buf = torch.zeros(1, device=self.device)
        self._host_loss = torch.zeros(1).pin_memory() if self.device.type == "cuda" else torch.zeros(1)
        self._staging: dict[int, torch.Tensor] = {}

    # ------------------------------------------------------------------
    def _inner(self):
        return getattr(self.model, "module", self.model)

    def compute_loss(self, batch: dict[str, torch.Tensor]):
        inner = self._inner()
        tc = self.config.train
        if self.bpr is not None:
            preds, cross = inner.forward_with_cross_scores(batch, cross_task=self.tasks[0])
            total, task_losses = self.loss_fn(preds, {t: batch[t] for t in self.tasks})
            bpr = self.bpr(cross, batch[self.tasks[0]])
            task_losses["bpr"] = bpr
            return total + tc.contrastive_weight * bpr, task_losses
        if hasattr(inner, "forward_loss") and tc.kernels == "native":
            total, task_losses, _ = inner.forward_loss(batch, tc.loss_weights, tc.regression_tasks)
            return total, task_losses
        preds = self.model(batch)
        return self.loss_fn(preds, {t: batch[t] for t in self.tasks if t in batch})

    def step(self, batch: dict[str, torch.Tensor]):
        """One optimisation step on a device-resident batch.
        Returns (detached loss tensor, {task: loss tensor})."""
        tc = self.config.train
        if self.sparse_opt is not None:
            self.sparse_opt.lr_scale = tc.sparse_warmup_value if self.global_step < tc.sparse_warmup_steps else 1.0
        self.model.train()
        self._zero_grad()
        with phase("pd.forward"), torch.autocast(self.device.type, dtype=torch.bfloat16, enabled=self.use_amp):
            total, task_losses = self.compute_loss(batch)
        # dense gradient sync overlapped with the backward: buckets of the flat
        # gradient arena are all-reduced as soon as their last gradient is written
        bucketed = self._bucketed_sync()
        overlapped = bucketed is not None and bucketed.begin()
        with phase("pd.backward"):
            total.backward()
        if self.grad_sync is not None and not self.fsdp:
            with phase("pd.dense_sync"):
                if not (overlapped and bucketed.finish()):
                    self.grad_sync.sync(self.flat.grad)
        with phase("pd.optimizer"):
            if tc.nan_guard and not bool(torch.isfinite(total)):
                self.skipped_steps += 1
            elif getattr(self.grad_sync, "sharded", False) and isinstance(self.optimizer, FusedAdamW):
                self.optimizer.step(shard=self.grad_sync.shard_range(self.flat.numel), group=self.grad_sync.group)
                self.grad_sync.gather_params(self.flat.data)
            else:
                self.optimizer.step()
        self.scheduler.step()
        self.global_step += 1
        return total.detach(), task_losses

    def _zero_grad(self) -> None:
        if self.flat is not None:
            self.flat.zero_grad()
        else:
            self.optimizer.zero_grad(set_to_none=True)

    def full_optimizer_state(self) -> dict:
        """The dense optimizer state with every shard gathered (collective
        when the state is sharded: every rank calls it)."""
        opt = self.optimizer
        if hasattr(opt, "full_state_dict"):
            return opt.full_state_dict()
        sd = opt.state_dict()
        if getattr(self.grad_sync, "sharded", False) and isinstance(opt, FusedAdamW):
            # zero2: each rank's moments are valid on its own slice only
            from primus_dlrm_b200.parallel.wrapper import all_gather_slices
            for k in ("exp_avg", "exp_avg_sq"):
                t = getattr(opt, k).clone()
                all_gather_slices(t, self.grad_sync.group)
                sd[k] = t.cpu()
        return sd

    def _bucketed_sync(self):
        """The peer-memory gradient sync when its per-bucket overlap with the
        backward is on (``PD_OVERLAP_DENSE_SYNC=0``: one all-reduce after the
        backward instead)."""
        gs = self.grad_sync
        if gs is None or os.environ.get("PD_OVERLAP_DENSE_SYNC", "1") == "0":
            return None
        impl = getattr(gs, "impl", None) or gs
        return impl if hasattr(impl, "begin") and hasattr(impl, "finish") else None

    def step_host(self, packed: PackedBatch) -> float:
        """End-to-end step through the public API: pinned host batch -> H2D
        copy -> step -> loss read back to the host."""
        buf = self._staging.get(packed.nbytes)
        if buf is None:
            buf = torch.empty(packed.nbytes, dtype=torch.uint8, device=self.device)
            self._staging[packed.nbytes] = buf
        batch = packed.to_device(self.device, out=buf)
        loss, _ = self.step(batch)
        self._host_loss.copy_(loss.reshape(1), non_blocking=True)
        if self.device.type == "cuda":
            torch.cuda.current_stream(self.device).synchronize()
        return float(self._host_loss[0])

    def exposed_comm_ms(self) -> float:
        """Device time of the embedding lookup + exchange since the last call."""
        inner = self._inner()
        ex = getattr(getattr(inner, "emb", None), "executor", None)
        return ex.take_comm_ms() if ex is not None and hasattr(ex, "take_comm_ms") else 0.0

    def state_dict(self) -> dict:
        return {"optimizer": self.full_optimizer_state(), "scheduler": self.scheduler.state_dict(),
                "global_step": self.global_step}

    def load_state_dict(self, sd: dict) -> None:
        self.optimizer.load_state_dict(sd["optimizer"])
        self.scheduler.load_state_dict(sd["scheduler"])
        self.global_step = int(sd.get("global_step", 0))


def _make_shampoo(params, tc):
    """Distributed Shampoo over the dense parameters (optional dependency
    ``distributed_shampoo``; settings as ``primus_dlrm/training/dist_trainer.py:175-230``):
    AdaGrad grafting, root-inverse preconditioner (bf16 factor matrices with an
    eigendecomposition when ``shampoo_use_bf16_factor_matrix``), the DDP
    distributed config when ``shampoo_use_ddp_distributed_config``, and the
    momentum / Nesterov / decoupled-weight-decay switches where the installed
    version accepts them."""
    try:
        import inspect

        from distributed_shampoo import DistributedShampoo
        from distributed_shampoo.shampoo_types import (AdaGradPreconditionerConfig, DDPDistributedConfig,
                                                       RootInvShampooPreconditionerConfig)
    except ImportError as e:
        raise RuntimeError("dense_optimizer='shampoo' needs the distributed_shampoo package "
                           "(facebookresearch/optimizers), which is not installed") from e
    if tc.shampoo_use_bf16_factor_matrix:
        from distributed_shampoo.preconditioner.matrix_functions_types import EigenConfig
        precond = RootInvShampooPreconditionerConfig(amortized_computation_config=EigenConfig(),
                                                     factor_matrix_dtype=torch.bfloat16,
                                                     inverse_exponent_override={1: 0.5, 2: 0.5},
                                                     num_tolerated_failed_amortized_computations=0)
    else:
        precond = RootInvShampooPreconditionerConfig()
    kw = dict(lr=tc.lr, betas=(0.9, 1.0), epsilon=1e-4, weight_decay=tc.weight_decay,
              max_preconditioner_dim=tc.shampoo_max_preconditioner_dim,
              precondition_frequency=tc.shampoo_precondition_frequency,
              start_preconditioning_step=tc.shampoo_precondition_frequency,
              grafting_config=AdaGradPreconditionerConfig(epsilon=1.0 / 70000.0),
              preconditioner_config=precond)
    if tc.shampoo_use_ddp_distributed_config:
        kw["distributed_config"] = DDPDistributedConfig(num_trainers_per_group=tc.shampoo_ddp_num_trainers_per_group,
                                                        communicate_params=tc.shampoo_ddp_communicate_params)
    accepted = inspect.signature(DistributedShampoo.__init__).parameters
    for key, val in (("momentum", tc.shampoo_momentum), ("use_nesterov", tc.shampoo_use_nesterov),
                     ("use_bias_correction", True),
                     ("use_decoupled_weight_decay", tc.shampoo_use_decoupled_weight_decay)):
        if key in accepted:
            kw[key] = val
    return DistributedShampoo(params, **kw)

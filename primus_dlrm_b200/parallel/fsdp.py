"""Fully sharded dense parameters (``distributed.dense_strategy: fsdp``).

The reference wraps the whole model in torch FSDP (one unit, fp32,
``use_orig_params``; ``primus_dlrm/distributed/wrapper.py:66-69``) and saves
full-state checkpoints gathered on rank 0
(``primus_dlrm/training/dist_trainer.py:729-739``). Here:

* every dense parameter is sharded along dim 0 over the ranks (FSDP2
  ``fully_shard``; the all-gathers and reduce-scatters are NCCL collectives,
  which use NVLS on NVSwitch): each rank stores 1/W of the fp32 master
  weights, of their gradients and of the AdamW moments (``ShardedAdamW``);
* every transformer block is its own unit and the rest of the model the root
  unit, so the full weights of at most two blocks exist at a time: a block's
  shards are all-gathered in the compute dtype (bf16 under ``train.bf16``)
  while the previous block computes, freed after its forward, gathered again
  (one block ahead) in the backward, and its gradients reduce-scattered in
  fp32 as soon as its backward ends;
* embedding tables stay on the sparse path (planner sharding, fused sparse
  optimizer, peer exchange) and are ignored by FSDP.

Weight gradients reach FSDP in the parameter dtype of the unsharded weights
(bf16 under ``train.bf16``) and are reduced in fp32.
"""
from __future__ import annotations

import math
from contextlib import contextmanager

import torch
import torch.distributed as dist
import torch.nn as nn

from primus_dlrm_b200.ops import _ext

try:
    from torch.distributed.device_mesh import DeviceMesh
    from torch.distributed.fsdp import FSDPModule, MixedPrecisionPolicy, fully_shard, register_fsdp_forward_method
    from torch.distributed.tensor import DTensor
except ImportError:          # pragma: no cover - torch without FSDP2
    fully_shard = None
    DTensor = ()
    FSDPModule = ()


def _local(t: torch.Tensor) -> torch.Tensor:
    return t.to_local() if isinstance(t, DTensor) else t


class FSDPSync:
    """What ``wrap_model`` returns for ``fsdp``: gradients are reduced by FSDP
    inside the backward, so the engine's explicit sync is a no-op."""

    fsdp = True
    sharded = False

    def __init__(self, group, mesh):
        self.group = group
        self.mesh = mesh

    def sync(self, *_args) -> None:
        return None

    def check(self) -> None:
        return None


def shard_dense(model: nn.Module, device: torch.device, group=None,
                compute_dtype: torch.dtype | None = None) -> FSDPSync:
    """Shard ``model``'s dense parameters in place (see module docstring)."""
    if fully_shard is None:
        raise RuntimeError("dense_strategy 'fsdp' needs torch.distributed.fsdp.fully_shard (FSDP2)")
    inner = getattr(model, "module", model)
    mesh = DeviceMesh.from_group(group if group is not None else dist.group.WORLD, device.type)
    # inputs are not cast at unit boundaries: autocast picks the compute dtype,
    # and the root's input is the whole batch (labels included)
    mp = MixedPrecisionPolicy(param_dtype=compute_dtype, reduce_dtype=torch.float32, cast_forward_inputs=False)
    emb = getattr(inner, "emb", None)
    ignored = set(emb.parameters()) if emb is not None else set()
    blocks = list(getattr(inner, "blocks", None) or [])
    for b in blocks:
        fully_shard(b, mesh=mesh, mp_policy=mp, reshard_after_forward=True)
    fully_shard(inner, mesh=mesh, mp_policy=mp, reshard_after_forward=False, ignored_params=ignored or None)
    for name in ("forward_loss", "forward_with_cross_scores"):
        if hasattr(inner, name):
            register_fsdp_forward_method(inner, name)
    for i in range(len(blocks) - 1):
        blocks[i].set_modules_to_forward_prefetch([blocks[i + 1]])
    for i in range(1, len(blocks)):
        blocks[i].set_modules_to_backward_prefetch([blocks[i - 1]])
    return FSDPSync(group, mesh)


def is_fsdp(model: nn.Module) -> bool:
    return bool(FSDPModule) and any(isinstance(m, FSDPModule) for m in model.modules())


@contextmanager
def full_params(model: nn.Module):
    """Every FSDP unit's full parameters for the duration of the block (paths
    such as the cached-S candidate scorer read block weights without calling
    the block). A no-op for an unsharded model."""
    mods = [m for m in model.modules() if isinstance(m, FSDPModule)] if FSDPModule else []
    for m in mods:
        m.unshard()
    try:
        yield
    finally:
        for m in mods:
            m.reshard()


def local_chunk(full: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    """This rank's dim-0 chunk of ``full`` for the sharded tensor ``like``
    (FSDP2 shards with ``torch.chunk`` semantics); ``full`` itself when
    ``like`` is not sharded."""
    if not isinstance(like, DTensor):
        return full
    mesh = like.device_mesh
    rank, world = mesh.get_local_rank(), mesh.size()
    chunks = torch.chunk(full, world, dim=0)
    out = chunks[rank] if rank < len(chunks) else full[:0]
    loc = like.to_local()
    if tuple(out.shape) != tuple(loc.shape):
        raise RuntimeError(f"shard shape {tuple(loc.shape)} does not match chunk {tuple(out.shape)} of "
                           f"{tuple(full.shape)}")
    return out


def full_tensor(t: torch.Tensor) -> torch.Tensor:
    """The unsharded value (collective for a DTensor: every rank calls it)."""
    return t.full_tensor() if isinstance(t, DTensor) else t


class ShardedAdamW(torch.optim.Optimizer):
    """AdamW with global-norm clipping over FSDP-sharded parameters: each rank
    updates its own shards (``_C.adamw_step`` per parameter on CUDA) with
    moments of the shard's size; the clip norm is the all-reduced sum of the
    shards' squared norms. Parameters FSDP ignores (replicated) get their
    gradients averaged here and enter the norm once.

    Semantics: ``torch.nn.utils.clip_grad_norm_`` + ``torch.optim.AdamW``
    (``primus_dlrm/training/dist_trainer.py:233,451-454``)."""

    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 1e-2, max_grad_norm: float = 0.0, group=None):
        super().__init__(list(params), dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        self.group = group
        self.max_grad_norm = max_grad_norm
        self.step_count = 0
        self.plist = [p for g in self.param_groups for p in g["params"]]
        self.exp_avg = [torch.zeros_like(_local(p), dtype=torch.float32) for p in self.plist]
        self.exp_avg_sq = [torch.zeros_like(_local(p), dtype=torch.float32) for p in self.plist]
        dev = _local(self.plist[0]).device
        self._sqnorm = torch.zeros(1, dtype=torch.float32, device=dev)
        self.native = _ext.native_enabled(dev)
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0

    @staticmethod
    def _aligned(t: torch.Tensor) -> bool:
        return t.is_contiguous() and t.dtype == torch.float32 and t.data_ptr() % 16 == 0

    def zero_grad(self, set_to_none: bool = True) -> None:
        for p in self.plist:
            p.grad = None

    @torch.no_grad()
    def step(self, closure=None):
        g0 = self.param_groups[0]
        lr, (b1, b2), eps, wd = g0["lr"], g0["betas"], g0["eps"], g0["weight_decay"]
        self.step_count += 1
        bc1, bc2 = 1 - b1 ** self.step_count, 1 - b2 ** self.step_count
        items = []
        for p, m, v in zip(self.plist, self.exp_avg, self.exp_avg_sq):
            if p.grad is None:
                continue
            g = _local(p.grad)
            if not isinstance(p, DTensor) and self.world > 1:
                dist.all_reduce(g, group=self.group)
                g.mul_(1.0 / self.world)
            items.append((_local(p), g, m, v, isinstance(p, DTensor)))
        clip = self.max_grad_norm > 0
        if clip:
            self._sqnorm.zero_()
            for p_l, g, _, _, sharded in items:
                if g.numel() == 0 or (not sharded and self.rank != 0):
                    continue
                if self.native and self._aligned(g):
                    _ext.core().grad_sqnorm(g, self._sqnorm)
                else:
                    self._sqnorm.add_(g.float().pow(2).sum())
            if self.world > 1:
                dist.all_reduce(self._sqnorm, group=self.group)
        for p_l, g, m, v, _ in items:
            if p_l.numel() == 0:
                continue
            if self.native and self._aligned(p_l):
                g32 = g if self._aligned(g) else g.float().contiguous().clone()
                _ext.core().adamw_step(p_l, g32, m, v, lr, b1, b2, eps, wd, bc1, bc2, self.max_grad_norm,
                                       self._sqnorm if clip else None)
                continue
            grad = g.float()
            if clip:
                grad = grad * torch.clamp(self.max_grad_norm / (self._sqnorm.sqrt() + 1e-6), max=1.0)
            p_l.mul_(1 - lr * wd)
            m.mul_(b1).add_(grad, alpha=1 - b1)
            v.mul_(b2).addcmul_(grad, grad, value=1 - b2)
            p_l.addcdiv_(m, (v.sqrt() / math.sqrt(bc2)).add_(eps), value=-lr / bc1)
        return None

    def _as_param(self, p: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        if isinstance(p, DTensor):
            return DTensor.from_local(t, p.device_mesh, p.placements, shape=p.shape, stride=p.stride())
        return t

    def full_state_dict(self, dst: int = 0) -> dict:
        """Unsharded moments (collective: every rank calls it). Each moment is
        gathered one parameter at a time on the device; only ``dst`` keeps the
        CPU copies (other ranks get ``None`` entries), so no rank but ``dst``
        holds the full optimizer state in host memory."""
        keep = self.rank == dst

        def gather(p, t):
            full = full_tensor(self._as_param(p, t))
            return full.cpu() if keep else None
        ea = [gather(p, m) for p, m in zip(self.plist, self.exp_avg)]
        es = [gather(p, v) for p, v in zip(self.plist, self.exp_avg_sq)]
        return {"step": self.step_count, "exp_avg": ea, "exp_avg_sq": es,
                "param_groups": [{k: v for k, v in g.items() if k != "params"} for g in self.param_groups]}

    def state_dict(self) -> dict:
        return self.full_state_dict()

    def load_state_dict(self, sd) -> None:
        self.step_count = int(sd["step"])
        for p, m, v, fm, fv in zip(self.plist, self.exp_avg, self.exp_avg_sq, sd["exp_avg"], sd["exp_avg_sq"]):
            m.copy_(local_chunk(fm.reshape(p.shape), p).to(m.device))
            v.copy_(local_chunk(fv.reshape(p.shape), p).to(v.device))
        for g, s in zip(self.param_groups, sd.get("param_groups", [])):
            g.update({k: v for k, v in s.items() if k in ("lr", "betas", "eps", "weight_decay", "initial_lr")})

"""Dense parameters in one flat fp32 arena + fused clip/AdamW.

All dense parameters of a model are re-homed as views of one contiguous
fp32 buffer, and their gradients as views of a second one.  This turns
the optimizer into one elementwise launch (``_C.adamw_step``), the global
gradient norm into one reduction (``_C.grad_sqnorm``), and the data-parallel
gradient sync into collectives over slices of one buffer.

Semantics: ``torch.nn.utils.clip_grad_norm_`` + ``torch.optim.AdamW``
(``primus_dlrm/training/dist_trainer.py:233,451-454``).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from primus_dlrm_b200.ops import _ext

_ALIGN = 64  # elements (256 B): keeps every parameter view 16-byte aligned


class FlatParams:
    """Re-home ``params`` into one flat buffer; grads become views of another."""

    def __init__(self, params: list[nn.Parameter]):
        self.params = [p for p in params if p.requires_grad]
        if not self.params:
            raise ValueError("FlatParams needs at least one trainable parameter")
        dev = self.params[0].device
        self.offsets = []
        n = 0
        for p in self.params:
            self.offsets.append(n)
            n += (p.numel() + _ALIGN - 1) // _ALIGN * _ALIGN
        self.numel = n
        self.data = torch.zeros(n, dtype=torch.float32, device=dev)
        self.grad = torch.zeros(n, dtype=torch.float32, device=dev)
        for p, off in zip(self.params, self.offsets):
            view = self.data[off:off + p.numel()].view_as(p)
            view.copy_(p.data)
            p.data = view
            p.grad = self.grad[off:off + p.numel()].view_as(p)

    def zero_grad(self) -> None:
        self.grad.zero_()
        for p, off in zip(self.params, self.offsets):
            g = p.grad
            if g is None or g.data_ptr() != self.grad[off:].data_ptr():
                p.grad = self.grad[off:off + p.numel()].view_as(p)

    def rebind_all(self) -> None:
        """Re-point every param's data at ``self.data`` (after the arena moved)."""
        for p, off in zip(self.params, self.offsets):
            p.data = self.data[off:off + p.numel()].view_as(p)

    def rebind(self) -> None:
        """Re-point params at the arena (after e.g. ``load_state_dict`` replaced data)."""
        for p, off in zip(self.params, self.offsets):
            view = self.data[off:off + p.numel()].view_as(p)
            if p.data.data_ptr() != view.data_ptr():
                view.copy_(p.data)
                p.data = view


class FusedAdamW(torch.optim.Optimizer):
    """AdamW over a ``FlatParams`` arena, with optional global-norm clipping.

    Exposes ``param_groups`` (one group, ``lr``) so torch LR schedulers work.
    ``state_dict()`` holds the flat moments and the step count.
    """

    def __init__(self, flat: FlatParams, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 1e-2, max_grad_norm: float = 0.0):
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
        super().__init__(flat.params, defaults)
        self.flat = flat
        self.max_grad_norm = max_grad_norm
        self.exp_avg = torch.zeros_like(flat.data)
        self.exp_avg_sq = torch.zeros_like(flat.data)
        self._sqnorm = torch.zeros(1, dtype=torch.float32, device=flat.data.device)
        self.step_count = 0
        self.native = _ext.native_enabled(flat.data.device)

    def grad_norm(self) -> torch.Tensor:
        """Global L2 norm of the flat gradient (device tensor, no sync)."""
        if self.native:
            self._sqnorm.zero_()
            _ext.core().grad_sqnorm(self.flat.grad, self._sqnorm)
            return self._sqnorm.sqrt()
        return self.flat.grad.norm()

    @torch.no_grad()
    def step(self, closure=None, shard: tuple[int, int] | None = None, group=None):
        """Update all parameters, or only the flat slice ``shard = (a, b)``
        (ZeRO-style sharded optimizer: the global gradient norm for clipping
        is then all-reduced over ``group``)."""
        g = self.param_groups[0]
        lr, (b1, b2), eps, wd = g["lr"], g["betas"], g["eps"], g["weight_decay"]
        self.step_count += 1
        bc1 = 1 - b1 ** self.step_count
        bc2 = 1 - b2 ** self.step_count
        f = self.flat
        a, b = shard if shard is not None else (0, f.numel)
        p, gr, m, v = f.data[a:b], f.grad[a:b], self.exp_avg[a:b], self.exp_avg_sq[a:b]
        if self.max_grad_norm > 0:
            if self.native:
                self._sqnorm.zero_()
                _ext.core().grad_sqnorm(gr, self._sqnorm)
            else:
                self._sqnorm.copy_(gr.float().pow(2).sum().reshape(1))
            if shard is not None:
                torch.distributed.all_reduce(self._sqnorm, group=group)
        if self.native:
            _ext.core().adamw_step(p, gr, m, v, lr, b1, b2, eps, wd, bc1, bc2, self.max_grad_norm,
                                   self._sqnorm if self.max_grad_norm > 0 else None)
            return None
        grad = gr
        if self.max_grad_norm > 0:
            coef = torch.clamp(self.max_grad_norm / (self._sqnorm.sqrt() + 1e-6), max=1.0)
            grad = grad * coef
        p.mul_(1 - lr * wd)
        m.mul_(b1).add_(grad, alpha=1 - b1)
        v.mul_(b2).addcmul_(grad, grad, value=1 - b2)
        denom = (v.sqrt() / math.sqrt(bc2)).add_(eps)
        p.addcdiv_(m, denom, value=-lr / bc1)
        return None

    def state_dict(self):
        return {"step": self.step_count, "exp_avg": self.exp_avg.cpu(), "exp_avg_sq": self.exp_avg_sq.cpu(),
                "param_groups": [{k: v for k, v in g.items() if k != "params"} for g in self.param_groups]}

    def load_state_dict(self, sd):
        self.step_count = int(sd["step"])
        self.exp_avg.copy_(sd["exp_avg"])
        self.exp_avg_sq.copy_(sd["exp_avg_sq"])
        for g, s in zip(self.param_groups, sd.get("param_groups", [])):
            g.update({k: v for k, v in s.items() if k in ("lr", "betas", "eps", "weight_decay", "initial_lr")})

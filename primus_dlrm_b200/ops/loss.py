"""Fused multi-task heads + weighted BCE/MSE loss.

Equivalent to ``{t: Linear_t(h)}`` followed by ``MultiTaskLoss``
(``primus_dlrm/training/losses.py:13-50``): BCE-with-logits for
classification tasks, MSE for ``regression_tasks``, weighted sum.
Native path: ``_C.heads_loss_fwd`` computes logits, per-task losses and the
logit gradients in one launch; ``_C.heads_loss_bwd`` produces dh, dW, db.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from primus_dlrm_b200.ops import _ext


class _HeadsLossFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, W, b, labels, task_weights, regression):
        C = _ext.core()
        # the kernel keeps the head weights in fp32 (FSDP may hand them over in bf16)
        ctx.wdt, ctx.bdt = W.dtype, b.dtype
        W, b = W.float().contiguous(), b.float().contiguous()
        out, logits, dlogit = C.heads_loss_fwd(h.contiguous(), W, b, labels.contiguous(), task_weights, regression)
        ctx.save_for_backward(h, W, dlogit)
        total = out[0]
        per_task = out[1:]
        ctx.mark_non_differentiable(per_task, logits)
        return total, per_task, logits

    @staticmethod
    def backward(ctx, g_total, _g_task, _g_logits):
        C = _ext.core()
        h, W, dlogit = ctx.saved_tensors
        if g_total is None:
            g_total = torch.zeros((), device=h.device)
        dh, dW, db = C.heads_loss_bwd(h.contiguous(), W.contiguous(), dlogit, g_total.reshape(1))
        return dh, dW.to(ctx.wdt), db.to(ctx.bdt), None, None, None


def heads_loss_ref(h, W, b, labels, task_weights, regression):
    logits = (h.float() @ W.float().t() + b.float()).t()  # [T, B]
    per = []
    for t in range(W.shape[0]):
        if regression[t]:
            per.append(F.mse_loss(logits[t], labels[t].float()))
        else:
            per.append(F.binary_cross_entropy_with_logits(logits[t], labels[t].float()))
    per_t = torch.stack(per)
    total = (per_t * torch.tensor(task_weights, device=per_t.device, dtype=per_t.dtype)).sum()
    return total, per_t, logits


def heads_loss(h: torch.Tensor, W: torch.Tensor, b: torch.Tensor, labels: torch.Tensor,
               task_weights: list[float], regression: list[int]):
    """h [B, D]; W [T, D]; b [T]; labels [T, B] -> (total, per_task [T], logits [T, B])."""
    if h.is_cuda and h.dtype == torch.bfloat16 and _ext.native_enabled(h.device) and W.shape[0] <= 16:
        return _HeadsLossFn.apply(h, W, b, labels, [float(x) for x in task_weights],
                                  [int(x) for x in regression])
    return heads_loss_ref(h, W, b, labels, task_weights, regression)

"""RMSNorm / LayerNorm (optionally fused with the residual add that feeds them).

Native path: ``_C.norm_fwd`` / ``_C.norm_bwd`` (one warp per row, bf16 in/out,
fp32 statistics).  Eager path: the reference formula
``(x.float() * rsqrt(mean(x^2) + eps)).to(x.dtype) * w``
(``primus_dlrm/models/onetrans.py:74-82``), which is also the test oracle.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from primus_dlrm_b200.ops import _ext


def _rows_ok(t: torch.Tensor) -> bool:
    """[B, R, D] view with contiguous, 16-byte aligned rows (any batch stride)."""
    return (t.dim() == 3 and t.stride(2) == 1 and (t.shape[1] == 1 or t.stride(1) == t.shape[2])
            and t.data_ptr() % 16 == 0 and t.stride(0) % 8 == 0) or t.is_contiguous()


def _f32(t: torch.Tensor | None) -> torch.Tensor | None:
    """Norm parameters as the kernels take them: contiguous fp32 (FSDP may hand
    them over in bf16; the gradient is cast back to the parameter's dtype)."""
    return t if t is None or (t.dtype == torch.float32 and t.is_contiguous()) else t.float().contiguous()


def _use_native(x: torch.Tensor) -> bool:
    return x.is_cuda and x.dtype == torch.bfloat16 and _ext.native_enabled(x.device) \
        and x.shape[-1] % 8 == 0 and x.shape[-1] <= 2048


class _NormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, res, weight, bias, eps: float, kind: int):
        C = _ext.core()
        xc = x if _rows_ok(x) else x.contiguous()
        rc = (res if _rows_ok(res) else res.contiguous()) if res is not None else None
        ctx.pdt = (weight.dtype, bias.dtype if bias is not None else None)
        weight, bias = _f32(weight), _f32(bias)
        y, z, rstd, mean = C.norm_fwd(xc, rc, weight, bias, eps, kind)
        xin = z if res is not None else xc
        if res is None and not xin.is_contiguous():
            xin = xin.contiguous()
        ctx.kind = kind
        ctx.fused = res is not None
        ctx.has_bias = bias is not None
        ctx.save_for_backward(xin, weight, rstd, mean if kind == 1 else rstd)
        if res is not None:
            return y, z
        return y

    @staticmethod
    def backward(ctx, *grads):
        C = _ext.core()
        xin, weight, rstd, mean = ctx.saved_tensors
        if ctx.fused:
            dy, dz = grads
        else:
            (dy,), dz = grads, None
        if dy is None:
            dy = torch.zeros_like(xin)
        dx, dw, db = C.norm_bwd(xin, dy.to(torch.bfloat16), dz.to(torch.bfloat16) if dz is not None else None,
                                weight, rstd, mean if ctx.kind == 1 else None, ctx.kind)
        dw, db = dw.to(ctx.pdt[0]), (db.to(ctx.pdt[1]) if ctx.has_bias else None)
        return (dx, dx if ctx.fused else None, dw, db, None, None)


class _NormTailFn(torch.autograd.Function):
    """``(norm(x), x[:, T - q:])`` as one autograd node.  A pre-norm block
    normalises all T rows of its input but carries only the last q rows on as
    the residual; with the slice taken here its gradient is added inside the
    norm backward kernel, so no zero-filled [B, T, D] gradient of the slice and
    no separate add are materialised."""

    @staticmethod
    def forward(ctx, x, weight, bias, eps: float, kind: int, q_len: int):
        C = _ext.core()
        xc = x if x.is_contiguous() else x.contiguous()
        ctx.pdt = (weight.dtype, bias.dtype if bias is not None else None)
        weight, bias = _f32(weight), _f32(bias)
        y, _, rstd, mean = C.norm_fwd(xc, None, weight, bias, eps, kind)
        T = x.shape[1]
        ctx.kind, ctx.has_bias, ctx.off = kind, bias is not None, T - q_len
        ctx.save_for_backward(xc, weight, rstd, mean if kind == 1 else rstd)
        return y, x[:, T - q_len:]

    @staticmethod
    def backward(ctx, dy, dtail):
        C = _ext.core()
        xin, weight, rstd, mean = ctx.saved_tensors
        if dy is None:
            dy = torch.zeros_like(xin)
        ex = dtail.to(torch.bfloat16) if dtail is not None else None
        dx, dw, db = C.norm_bwd(xin, dy.to(torch.bfloat16), ex, weight, rstd,
                                mean if ctx.kind == 1 else None, ctx.kind, ctx.off if ex is not None else 0)
        return dx, dw.to(ctx.pdt[0]), (db.to(ctx.pdt[1]) if ctx.has_bias else None), None, None, None


def norm_with_tail(norm: nn.Module, x: torch.Tensor, q_len: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(norm(x), x[:, T - q_len:]) for x [B, T, D]; one fused backward when native."""
    T = x.shape[1]
    if _use_native(x) and x.dim() == 3 and 0 < q_len <= T:
        return _NormTailFn.apply(x, norm.weight, getattr(norm, "bias", None), norm.eps, norm.kind, q_len)
    return norm(x), x[:, T - q_len:]


def rms_norm_ref(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    rms = x.float().pow(2).mean(-1, keepdim=True).add(eps).rsqrt()
    return (x.float() * rms).to(x.dtype) * weight


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    if _use_native(x):
        return _NormFn.apply(x, None, weight, None, eps, 0)
    return rms_norm_ref(x, weight, eps)


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    if _use_native(x):
        return _NormFn.apply(x, None, weight, bias, eps, 1)
    return torch.nn.functional.layer_norm(x.float(), (x.shape[-1],), weight, bias, eps).to(x.dtype)


def add_norm(a: torch.Tensor, b: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
             eps: float, kind: int) -> tuple[torch.Tensor, torch.Tensor]:
    """z = a + b; returns (norm(z), z) with one pass over memory when native."""
    if _use_native(a) and b.dtype == a.dtype and b.shape == a.shape and a.dim() == 3:
        y, z = _NormFn.apply(a, b, weight, bias, eps, kind)
        return y, z
    z = a + b
    if kind == 0:
        return rms_norm_ref(z, weight, eps), z
    return torch.nn.functional.layer_norm(z.float(), (z.shape[-1],), weight, bias, eps).to(z.dtype), z


class RMSNorm(nn.Module):
    """Same parameters and state-dict key (``weight``) as the reference module."""

    def __init__(self, d: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))
        self.eps = eps
        self.kind = 0

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return rms_norm(x, self.weight, self.eps)


class LayerNorm(nn.Module):
    def __init__(self, d: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))
        self.bias = nn.Parameter(torch.zeros(d))
        self.eps = eps
        self.kind = 1

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return layer_norm(x, self.weight, self.bias, self.eps)


def make_norm(kind: str, d: int) -> nn.Module:
    if kind == "rmsnorm":
        return RMSNorm(d)
    if kind == "layernorm":
        return LayerNorm(d)
    raise ValueError(f"unknown norm {kind!r} (rmsnorm | layernorm)")

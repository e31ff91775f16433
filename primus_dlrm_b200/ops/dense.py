"""Dense projections of the OneTrans / DLRM stacks.

``mixed_linear`` is the mixed-parameterisation projection of
``primus_dlrm/models/onetrans.py:124-134,196-204``: rows ``[:n_s]`` of every
sample share ``W_s``; NS row ``n_s + t`` uses its own ``W_ns[t]``.  The result
is one ``[B, T, D_out]`` tensor (the reference builds the S and NS parts
separately and concatenates them).

``mlp2`` is ``Linear -> GELU -> Linear`` (tokenizers).

When the ``_gemm`` extension is present these run on the sm_100a tcgen05
kernels (grouped GEMM with the NS tokens as extra groups, GELU fused in the
epilogue); otherwise PyTorch ops (cuBLAS under autocast / CPU) express the
same math.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from primus_dlrm_b200.ops import _ext


def _gemm_ok(x: torch.Tensor) -> bool:
    if not (x.is_cuda and _ext.native_enabled(x.device)):
        return False
    g = _ext.gemm()
    return g is not None and hasattr(g, "mixed_linear_fwd")


def _cast_w(w: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    return w.to(like.dtype) if w.dtype != like.dtype else w


class _MixedLinearNative(torch.autograd.Function):
    """tcgen05 grouped GEMM: one launch for the shared S rows + all NS tokens."""

    @staticmethod
    def forward(ctx, x, w_s, w_ns, n_s: int, act: str):
        G = _ext.gemm()
        xb = x.contiguous()
        wsb = w_s.to(torch.bfloat16)
        wnb = w_ns.to(torch.bfloat16)
        y, pre = G.mixed_linear_fwd(xb, wsb, wnb, n_s, act == "gelu")
        ctx.save_for_backward(xb, wsb, wnb, pre if act == "gelu" else y.new_empty(0))
        ctx.n_s, ctx.act = n_s, act
        ctx.w_dtypes = (w_s.dtype, w_ns.dtype)
        return y

    @staticmethod
    def backward(ctx, dy):
        G = _ext.gemm()
        xb, wsb, wnb, pre = ctx.saved_tensors
        dx, dws, dwn = G.mixed_linear_bwd(dy.contiguous().to(torch.bfloat16), xb, wsb, wnb,
                                          pre if ctx.act == "gelu" else None, ctx.n_s)
        return dx, dws.to(ctx.w_dtypes[0]), dwn.to(ctx.w_dtypes[1]), None, None


class _MixedLinearTorch(torch.autograd.Function):
    """Library-GEMM version with an explicit backward: the S GEMM runs over all
    T rows and the NS rows are overwritten in place, so neither direction
    materialises a concatenation or a zero-filled gradient copy."""

    @staticmethod
    def forward(ctx, x, w_s, w_ns, n_s: int, act: str):
        dt = x.dtype
        ws, wn = w_s.to(dt), w_ns.to(dt)
        y = torch.matmul(x, ws.t())
        if x.shape[1] > n_s:
            y[:, n_s:] = torch.einsum("btn,tmn->btm", x[:, n_s:], wn)
        pre = None
        if act == "gelu":
            pre = y
            y = F.gelu(pre)
        ctx.save_for_backward(x, ws, wn, pre if pre is not None else y.new_empty(0))
        ctx.n_s, ctx.act, ctx.wdt = n_s, act, (w_s.dtype, w_ns.dtype)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, ws, wn, pre = ctx.saved_tensors
        n_s = ctx.n_s
        dy = dy.to(x.dtype)
        if ctx.act == "gelu":
            dy = torch.ops.aten.gelu_backward(dy, pre)
        B, T, K = x.shape
        N = dy.shape[-1]
        dx = torch.matmul(dy, ws)
        dws = torch.matmul(dy.reshape(-1, N).t(), x.reshape(-1, K)).float()
        dwn = None
        if T > n_s:
            dy_ns, x_ns = dy[:, n_s:], x[:, n_s:]
            dx[:, n_s:] = torch.einsum("btm,tmn->btn", dy_ns, wn)
            dwn = torch.einsum("btm,btn->tmn", dy_ns.float(), x_ns.float())
            dws -= dwn.sum(0)
        else:
            dwn = torch.zeros(wn.shape, dtype=torch.float32, device=x.device)
        return dx, dws.to(ctx.wdt[0]), dwn.to(ctx.wdt[1]), None, None


def mixed_linear(x: torch.Tensor, n_s: int, w_s: torch.Tensor, w_ns: torch.Tensor,
                 act: str | None = None) -> torch.Tensor:
    """x [B, T, Din] -> [B, T, Dout]; rows < n_s use w_s [Dout, Din], row n_s+t uses w_ns[t]."""
    if _gemm_ok(x) and x.dtype == torch.bfloat16:
        return _MixedLinearNative.apply(x, w_s, w_ns, n_s, act or "")
    if x.is_cuda and x.dtype == torch.bfloat16:
        return _MixedLinearTorch.apply(x, w_s, w_ns, n_s, act or "")
    y = F.linear(x, w_s)
    if x.shape[1] > n_s:
        ns = torch.einsum("btn,tmn->btm", x[:, n_s:], w_ns)
        y[:, n_s:] = ns.to(y.dtype)
    if act == "gelu":
        y = F.gelu(y)
    return y


def mlp2(x: torch.Tensor, l1: nn.Linear, l2: nn.Linear) -> torch.Tensor:
    """l2(GELU(l1(x)))."""
    return l2(F.gelu(l1(x)))

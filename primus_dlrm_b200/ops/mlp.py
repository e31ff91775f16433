"""MLP chains and the low-rank DCNv2 cross layer on the tcgen05 GEMM (DLRM).

``mlp_chain`` runs ``Linear (+ ReLU)`` stacks (``make_mlp`` of
``primus_dlrm/models/interaction.py:10-18``): the bias and ReLU are fused into
each GEMM's epilogue, and in the backward the next layer's data-gradient GEMM
applies this layer's ReLU mask in its epilogue (the gradient leaves as the
pre-activation gradient), so no elementwise pass runs between layers.

``cross_layer`` is one low-rank DCNv2 cross layer,
``x_{l+1} = x0 * (x_l U V + b) + x_l`` (the full-rank form of
``primus_dlrm/models/interaction.py:98-140`` with ``W = U V``): ``t = x_l U``,
then one GEMM over ``[t | 1]`` and ``[V ; b]`` (the bias as an extra K row)
whose epilogue computes ``x0 * acc + x_l`` and stores ``acc`` for the
backward. The backward's ``dx_l = dy + (dy x0) V^T U^T`` adds ``dy`` in the
epilogue of its last GEMM.

Weight gradients run on the tcgen05 split-K kernel when their shapes allow
(both dims multiples of 64), else on ``torch.mm`` with fp32 output.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from primus_dlrm_b200.ops import _ext
from primus_dlrm_b200.ops.dense import tc_gemm, tc_wgrad

_EPI_RELU, _EPI_ADD = "relu", "residual"


def _bf(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)


def _rows(t: torch.Tensor) -> torch.Tensor:
    """[M, N] -> the [1, M, N] view the GEMM takes."""
    return t.reshape(1, t.shape[0], t.shape[1])


def _bias_rows(b: torch.Tensor, M: int) -> torch.Tensor:
    """A bias [N] as a [1, M, N] addend through zero strides."""
    return _bf(b).reshape(1, 1, -1).expand(1, M, b.numel())


def _wgrad(dy: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """dW = dy^T x in fp32 ([N, K] from dy [M, N], x [M, K])."""
    N, K = dy.shape[1], x.shape[1]
    if N % 64 == 0 and K % 64 == 0:
        return tc_wgrad(_rows(dy), _rows(x), torch.zeros(1, N, K, device=dy.device))[0]
    return torch.mm(dy.t(), x, out_dtype=torch.float32)


def _pad8(x: torch.Tensor) -> torch.Tensor:
    k = x.shape[-1]
    if k % 8 == 0:
        return x
    return torch.nn.functional.pad(x, (0, 8 - k % 8))


class _MLPChain(torch.autograd.Function):
    """h_i = act_i(h_{i-1} W_i^T + b_i) for i = 1..n, act in {relu, none}."""

    @staticmethod
    def forward(ctx, x, acts: tuple, *wb):
        ws, bs = wb[0::2], wb[1::2]
        k_in = x.shape[1]
        h = _pad8(_bf(x).contiguous())
        hs = [h]
        wbf = []
        for w, b, act in zip(ws, bs, acts):
            wb_ = _bf(w)
            if wb_.shape[1] != h.shape[1]:                 # the first layer's K padded to a multiple of 8
                wb_ = torch.nn.functional.pad(wb_, (0, h.shape[1] - wb_.shape[1]))
            wbf.append(wb_.contiguous())
            out = torch.empty(h.shape[0], w.shape[0], dtype=torch.bfloat16, device=x.device)
            tc_gemm(_rows(h), wbf[-1].reshape(1, *wbf[-1].shape), _rows(out),
                    _EPI_RELU if act == "relu" else _EPI_ADD, R=_bias_rows(b, h.shape[0]))
            h = out
            hs.append(h)
        ctx.save_for_backward(*hs, *wbf)
        ctx.acts, ctx.k_in, ctx.n = acts, k_in, len(ws)
        ctx.wdt = [t.dtype for t in wb]
        ctx.x_grad = x.requires_grad
        return h

    @staticmethod
    def backward(ctx, dout):
        n = ctx.n
        saved = ctx.saved_tensors
        hs, wbf = saved[: n + 1], saved[n + 1:]
        acts = ctx.acts
        d = _bf(dout).contiguous()
        if acts[-1] == "relu":
            d = torch.where(hs[-1] > 0, d, torch.zeros((), dtype=d.dtype, device=d.device))
        grads = [None] * (2 * n)
        dx = None
        for i in reversed(range(n)):
            gw = _wgrad(d, hs[i])
            if i == 0 and gw.shape[1] != ctx.k_in:            # drop the K padding of the first layer
                gw = gw[:, : ctx.k_in]
            grads[2 * i] = gw.to(ctx.wdt[2 * i])
            grads[2 * i + 1] = d.sum(0, dtype=torch.float32).to(ctx.wdt[2 * i + 1])
            if i > 0 or ctx.x_grad:
                K = wbf[i].shape[1]
                nxt = torch.empty(d.shape[0], K, dtype=torch.bfloat16, device=d.device)
                if K % 64 == 0:
                    # the data gradient, masked by the previous layer's ReLU in the epilogue
                    mask = i > 0 and acts[i - 1] == "relu"
                    tc_gemm(_rows(d), wbf[i].reshape(1, *wbf[i].shape), _rows(nxt), "mask_pos" if mask else None,
                            R=_rows(hs[i]) if mask else None, b_kn=True)
                else:
                    nxt = torch.mm(d, wbf[i])
                    if i > 0 and acts[i - 1] == "relu":
                        nxt = torch.where(hs[i] > 0, nxt, torch.zeros((), dtype=nxt.dtype, device=nxt.device))
                if i > 0:
                    d = nxt
                else:
                    dx = nxt[:, : ctx.k_in]
        return (dx, None, *grads)


def _chain_layers(seq: nn.Module):
    """(linears, acts) of a Linear / ReLU Sequential (make_mlp with dropout 0),
    or None when it holds anything else."""
    if not isinstance(seq, nn.Sequential):
        return None
    lins, acts = [], []
    for m in seq:
        if isinstance(m, nn.Linear):
            if m.bias is None:
                return None
            lins.append(m)
            acts.append(None)
        elif isinstance(m, nn.ReLU) and lins and acts[-1] is None:
            acts[-1] = "relu"
        elif isinstance(m, nn.Dropout) and (m.p == 0 or not m.training):
            continue
        else:
            return None
    return (lins, tuple(acts)) if lins else None


def native_ok(x: torch.Tensor) -> bool:
    return (x.is_cuda and _ext.native_enabled(x.device) and x.dtype == torch.bfloat16 and x.dim() == 2
            and _ext.gemm() is not None and hasattr(_ext.gemm(), "tc_gemm"))


def mlp_chain(seq: nn.Module, x: torch.Tensor) -> torch.Tensor:
    """``seq(x)`` for a Linear / ReLU stack, on the tcgen05 GEMM when the
    shapes allow (every output width a multiple of 64), else ``seq(x)``."""
    layers = _chain_layers(seq) if native_ok(x) else None
    if layers is None or any(m.out_features % 64 for m in layers[0]):
        return seq(x)
    lins, acts = layers
    wb = [t for m in lins for t in (m.weight, m.bias)]
    return _MLPChain.apply(x, acts, *wb)


def linear(lin: nn.Linear, x: torch.Tensor) -> torch.Tensor:
    """One Linear (+ bias) on the tcgen05 GEMM when the shapes allow."""
    if not native_ok(x) or lin.bias is None or lin.out_features % 64:
        return lin(x)
    return _MLPChain.apply(x, (None,), lin.weight, lin.bias)


class _Cross(torch.autograd.Function):
    """x_{l+1} = x0 * (x_l U V + b) + x_l; U [d, r], V [r, d], b [d]."""

    @staticmethod
    def forward(ctx, x0, xl, U, V, b):
        B, d = xl.shape
        r = U.shape[1]
        x0b, xlb = _bf(x0).contiguous(), _bf(xl).contiguous()
        ub, vb = _bf(U).contiguous(), _bf(V).contiguous()
        # [t | 1 | 0 ...]: t = x_l U written into the first r columns
        ta = torch.zeros(B, r + 8, dtype=torch.bfloat16, device=xl.device)
        ta[:, r] = 1.0
        tc_gemm(_rows(xlb), ub.reshape(1, d, r), _rows(ta[:, :r]), None, b_kn=True)
        # [V ; b ; 0 ...] read as [K, N]
        va = torch.zeros(r + 8, d, dtype=torch.bfloat16, device=xl.device)
        va[:r] = vb
        va[r] = _bf(b)
        y = torch.empty(B, d, dtype=torch.bfloat16, device=xl.device)
        pre = torch.empty_like(y)                                  # t V + b
        tc_gemm(_rows(ta), va.reshape(1, r + 8, d), _rows(y), "mul_add", R=_rows(x0b), AUX=_rows(pre),
                b_kn=True, R2=_rows(xlb))
        ctx.save_for_backward(x0b, xlb, ub, vb, ta, pre)
        ctx.wdt = (U.dtype, V.dtype, b.dtype)
        return y

    @staticmethod
    def backward(ctx, dy):
        x0b, xlb, ub, vb, ta, pre = ctx.saved_tensors
        r = ub.shape[1]
        dy = _bf(dy).contiguous()
        dx0 = dy * pre
        dp = dy * x0b
        B, d = dy.shape
        dt = torch.empty(B, r, dtype=torch.bfloat16, device=dy.device)
        tc_gemm(_rows(dp), vb.reshape(1, r, d), _rows(dt))                      # dp V^T
        dxl = torch.empty(B, d, dtype=torch.bfloat16, device=dy.device)
        tc_gemm(_rows(dt), ub.reshape(1, d, r), _rows(dxl), "residual", R=_rows(dy))   # dt U^T + dy
        t = ta[:, :r]
        dV = _wgrad_t(t, dp)
        dU = _wgrad_t(xlb, dt)
        db = dp.sum(0, dtype=torch.float32)
        return dx0, dxl, dU.to(ctx.wdt[0]), dV.to(ctx.wdt[1]), db.to(ctx.wdt[2])


def _wgrad_t(a: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
    """a^T g in fp32: [Ka, Kg] from a [M, Ka], g [M, Kg] (the weight gradient of
    a product ``a @ W``)."""
    Ka, Kg = a.shape[1], g.shape[1]
    if Ka % 64 == 0 and Kg % 64 == 0:
        return tc_wgrad(_rows(a), _rows(g), torch.zeros(1, Ka, Kg, device=a.device))[0]
    return torch.mm(a.t(), g, out_dtype=torch.float32)


def cross_ok(x: torch.Tensor, d: int, r: int) -> bool:
    return native_ok(x) and d % 64 == 0 and r % 64 == 0


def cross_layer(x0: torch.Tensor, xl: torch.Tensor, U: torch.Tensor, V: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return _Cross.apply(x0, xl, U, V, b)

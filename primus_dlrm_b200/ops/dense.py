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

import os

import torch
import torch.nn as nn
import torch.nn.functional as F

from primus_dlrm_b200.ops import _ext


def _gemm_ok(x: torch.Tensor) -> bool:
    if not (x.is_cuda and _ext.native_enabled(x.device)):
        return False
    g = _ext.gemm()
    return g is not None and hasattr(g, "tc_gemm")


def _cast_w(w: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    return w.to(like.dtype) if w.dtype != like.dtype else w


# gelu_d: GELU with its derivative stored in AUX; mul: acc * R (the backward
# through that stored derivative)
# relu: bias (R) + ReLU; mask_pos: acc where R > 0 (a ReLU layer's backward);
# mul_add: R * acc + R2 (the DCNv2 cross layer)
_EPI = {"": 0, None: 0, "gelu": 1, "residual": 2, "dgelu": 3, "gelu_d": 4, "mul": 5, "relu": 6, "mask_pos": 7,
        "mul_add": 8}
_err_words: dict = {}


def _err(device) -> torch.Tensor:
    e = _err_words.get(device)
    if e is None:
        e = torch.zeros(1, dtype=torch.int32, device=device)
        _err_words[device] = e
    return e


def gemm_error_code(device) -> int:
    """Error word of the tcgen05 GEMMs on ``device`` (2 = a pipeline wait timed out)."""
    e = _err_words.get(torch.device(device))
    return int(e.item()) if e is not None else 0


def tc_gemm(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, epi: str | None = None,
            R: torch.Tensor | None = None, AUX: torch.Tensor | None = None, b_kn: bool = False,
            R2: torch.Tensor | None = None) -> torch.Tensor:
    """C[l] = epi(A[l] @ B[l]^T) on the sm_100a tcgen05 kernel; A [L, M, K],
    B [L or 1, N, K] -- or with ``b_kn`` [L or 1, K, N], a weight used
    transposed, read in place -- C/R/AUX/R2 [L, M, N] (bf16 views, unit stride
    on the last dim)."""
    _ext.gemm().tc_gemm(A, B, C, _EPI[epi], R, AUX, _err(A.device), b_kn, R2)
    return C


def tc_wgrad(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, l_sum: bool = False) -> torch.Tensor:
    """C[l] (fp32 [M, N], zeroed) += A[l]^T B[l] summed over the rows on the
    tcgen05 kernel: A [L, K, M], B [L, K, N] bf16 views (the output gradient
    and the input of a projection, both as stored).  With ``l_sum`` C is
    [1, M, N] and the sum runs over the L batches too (e.g. the samples of a
    strided per-sample token range)."""
    _ext.gemm().tc_wgrad(A, B, C, _err(A.device), l_sum)
    return C


def _wgrad_ok(t: torch.Tensor, M: int, N: int) -> bool:
    """Weight gradients on the tcgen05 split-K kernel (default; PD_WGRAD_TC=0
    selects cuBLAS). These products stream dY and X once and are bound by HBM;
    the kernel measures within 1-6 % of cuBLAS's split-K GEMMs on the v6 shapes
    and writes fp32 straight from its accumulators."""
    g = _ext.gemm()
    return (hasattr(g, "tc_wgrad") and t.dtype == torch.bfloat16 and M % 64 == 0 and N % 64 == 0
            and os.environ.get("PD_WGRAD_TC", "1") != "0")


def _tc_ok(x: torch.Tensor, K: int, N: int) -> bool:
    return x.dtype == torch.bfloat16 and K % 8 == 0 and N % 64 == 0 and x.data_ptr() % 16 == 0


def _mixed_tc(x, n_s, ws, wn, out, epi=None, R=None, AUX=None, b_kn=False):
    """out = epi(mixed(x)) with the tcgen05 GEMM: all T rows with ws, then the
    NS rows (one batch per token) with wn.  x [B, T, K]; ws [N, K]; wn [NS, N, K]
    -- or with ``b_kn`` the forward weights ws [K, N], wn [NS, K, N] applied
    transposed (the data gradient), read in place."""
    Bsz, T, K = x.shape
    N = ws.shape[1] if b_kn else ws.shape[0]
    v = lambda t: t.reshape(1, Bsz * T, t.shape[-1]) if t is not None else None
    tc_gemm(v(x), ws.reshape(1, *ws.shape), v(out), epi, v(R), v(AUX), b_kn=b_kn)
    if T > n_s:
        tr = lambda t: t[:, n_s:].transpose(0, 1) if t is not None else None
        tc_gemm(tr(x), wn, tr(out), epi, tr(R), tr(AUX), b_kn=b_kn)
    return out


def _dw(dy, x, n_s, wdt):
    """Weight gradients of a mixed projection (cuBLAS): shared S weight from
    the first n_s rows of every sample, per-token NS weights."""
    B, T, N = dy.shape
    K = x.shape[-1]
    if _wgrad_ok(dy, N, K):
        # tcgen05, both operands as stored, split over the rows, fp32 out: the
        # S weight over every row as one flat product (one long split-K; the
        # S rows alone are 2048 short strided batches, which measured slower),
        # minus the NS rows' part, each NS weight over its token's rows
        dws = tc_wgrad(dy.reshape(1, -1, N), x.reshape(1, -1, K), torch.zeros(1, N, K, device=dy.device))[0]
        if T > n_s:
            dwn = tc_wgrad(dy[:, n_s:].transpose(0, 1), x[:, n_s:].transpose(0, 1),
                           torch.zeros(T - n_s, N, K, device=dy.device))
            dws -= dwn.sum(0)
        else:
            dwn = torch.zeros(0, N, K, device=dy.device)
        return dws.to(wdt[0]), dwn.to(wdt[1])
    # fp32 results straight from the GEMM (no bf16 round trip, no cast kernel)
    dws = torch.mm(dy.reshape(-1, N).t(), x.reshape(-1, K), out_dtype=torch.float32)
    if T > n_s:
        # one GEMM per NS token over the batch: [N, B] x [B, K] views, no copies
        dwn = torch.bmm(dy[:, n_s:].permute(1, 2, 0), x[:, n_s:].transpose(0, 1), out_dtype=torch.float32)
        dws -= dwn.sum(0)
    else:
        dwn = torch.zeros(0, N, K, device=dy.device)
    return dws.to(wdt[0]), dwn.to(wdt[1])


class _MixedLinearNative(torch.autograd.Function):
    """Mixed projection on the tcgen05 GEMM (GELU fused into the epilogue)."""

    @staticmethod
    def forward(ctx, x, w_s, w_ns, n_s: int, act: str):
        xb = x.contiguous()
        ws, wn = w_s.to(torch.bfloat16), w_ns.to(torch.bfloat16)
        B, T, _ = xb.shape
        N = ws.shape[0]
        y = torch.empty(B, T, N, dtype=torch.bfloat16, device=x.device)
        dact = torch.empty_like(y) if act == "gelu" else None       # GELU'(pre-activation)
        _mixed_tc(xb, n_s, ws, wn, y, "gelu_d" if act == "gelu" else None, AUX=dact)
        ctx.save_for_backward(xb, ws, wn, dact if dact is not None else y.new_empty(0))
        ctx.n_s, ctx.act, ctx.wdt = n_s, act, (w_s.dtype, w_ns.dtype)
        return y

    @staticmethod
    def backward(ctx, dy):
        xb, ws, wn, dact = ctx.saved_tensors
        dy = dy.contiguous().to(torch.bfloat16)
        if ctx.act == "gelu":
            dy = dy * dact
        B, T, K = xb.shape
        dx = torch.empty(B, T, K, dtype=torch.bfloat16, device=xb.device)
        _mixed_tc(dy, ctx.n_s, ws, wn, dx, b_kn=True)
        dws, dwn = _dw(dy, xb, ctx.n_s, ctx.wdt)
        return dx, dws, dwn, None, None


class MixedFFNNative(torch.autograd.Function):
    """out = z + W2(GELU(W1 x)) for the mixed S / NS parameterisation, on the
    tcgen05 GEMM: GELU fused into the up projection (which also stores GELU'
    of the pre-activation), the residual add into the down projection, and the
    product with GELU' into the down projection's data-gradient GEMM."""

    @staticmethod
    def forward(ctx, x, z, w1, w2, wn1, wn2, n_s: int):
        xb = x.contiguous()
        bw = [w.to(torch.bfloat16) for w in (w1, w2, wn1, wn2)]
        B, T, D = xb.shape
        F_ = bw[0].shape[0]
        h = torch.empty(B, T, F_, dtype=torch.bfloat16, device=x.device)
        dact = torch.empty_like(h)                                # GELU'(pre-activation)
        _mixed_tc(xb, n_s, bw[0], bw[2], h, "gelu_d", AUX=dact)
        out = torch.empty(B, T, D, dtype=torch.bfloat16, device=x.device)
        _mixed_tc(h, n_s, bw[1], bw[3], out, "residual", R=z)
        ctx.save_for_backward(xb, h, dact, *bw)
        ctx.n_s = n_s
        ctx.wdt = [w.dtype for w in (w1, w2, wn1, wn2)]
        return out

    @staticmethod
    def backward(ctx, dout):
        xb, h, dact, w1, w2, wn1, wn2 = ctx.saved_tensors
        n_s = ctx.n_s
        dout = dout.contiguous().to(torch.bfloat16)
        B, T, D = xb.shape
        F_ = w1.shape[0]
        dpre = torch.empty(B, T, F_, dtype=torch.bfloat16, device=xb.device)
        _mixed_tc(dout, n_s, w2, wn2, dpre, "mul", R=dact, b_kn=True)
        dw2, dwn2 = _dw(dout, h, n_s, (ctx.wdt[1], ctx.wdt[3]))
        dx = torch.empty(B, T, D, dtype=torch.bfloat16, device=xb.device)
        _mixed_tc(dpre, n_s, w1, wn1, dx, b_kn=True)
        dw1, dwn1 = _dw(dpre, xb, n_s, (ctx.wdt[0], ctx.wdt[2]))
        return dx, dout, dw1, dw2, dwn1, dwn2, None


def mixed_ffn(x: torch.Tensor, z: torch.Tensor, n_s: int, w1, w2, wn1, wn2) -> torch.Tensor | None:
    """Fused native FFN + residual, or None when the native GEMM cannot run it."""
    if not (_gemm_ok(x) and x.dtype == torch.bfloat16 and z.dtype == torch.bfloat16):
        return None
    D, F_ = w2.shape[0], w1.shape[0]
    if not (_tc_ok(x, D, F_) and F_ % 64 == 0 and D % 64 == 0 and z.stride(-1) == 1 and z.stride(-2) % 8 == 0):
        return None
    return MixedFFNNative.apply(x, z, w1, w2, wn1, wn2, n_s)


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
            dwn = torch.einsum("btm,btn->tmn", dy_ns, x_ns).float()
            dws -= dwn.sum(0)
        else:
            dwn = torch.zeros(wn.shape, dtype=torch.float32, device=x.device)
        return dx, dws.to(ctx.wdt[0]), dwn.to(ctx.wdt[1]), None, None


def mixed_linear(x: torch.Tensor, n_s: int, w_s: torch.Tensor, w_ns: torch.Tensor,
                 act: str | None = None) -> torch.Tensor:
    """x [B, T, Din] -> [B, T, Dout]; rows < n_s use w_s [Dout, Din], row n_s+t uses w_ns[t]."""
    if _gemm_ok(x) and _tc_ok(x, x.shape[-1], w_s.shape[0]):
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


class _LinearNative(torch.autograd.Function):
    """y = act(x W^T + b) on the tcgen05 GEMM, act in {none, gelu, relu}: the
    bias and activation in the epilogue (GELU' stored for the backward), the
    weight gradient on the split-K kernel. x [..., K] (K padded to a multiple
    of 64 inside, so the data gradient's GEMM runs on the same kernel), W [N, K]
    with N a multiple of 64."""

    @staticmethod
    def forward(ctx, x, w, b, act: str):
        K, N = w.shape[1], w.shape[0]
        lead = x.shape[:-1]
        x2 = x.reshape(-1, K).to(torch.bfloat16)
        wb = w.to(torch.bfloat16)
        if K % 64:
            x2 = F.pad(x2, (0, -K % 64))
            wb = F.pad(wb, (0, -K % 64))
        x2, wb = x2.contiguous(), wb.contiguous()
        M = x2.shape[0]
        y = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
        r = b.to(torch.bfloat16).reshape(1, 1, N).expand(1, M, N) if b is not None else None
        aux = torch.empty_like(y) if act == "gelu" else None
        epi = {"gelu": "gelu_d", "relu": "relu"}.get(act, "residual" if r is not None else None)
        tc_gemm(x2.reshape(1, M, -1), wb.reshape(1, N, -1), y.reshape(1, M, N), epi, R=r,
                AUX=aux.reshape(1, M, N) if aux is not None else None)
        ctx.save_for_backward(x2, wb, aux if act == "gelu" else (y if act == "relu" else y.new_empty(0)))
        ctx.meta = (act, K, lead, w.dtype, b.dtype if b is not None else None)
        return y.reshape(*lead, N)

    @staticmethod
    def backward(ctx, dy):
        x2, wb, saved = ctx.saved_tensors
        act, K, lead, wdt, bdt = ctx.meta
        N = wb.shape[0]
        d = dy.reshape(-1, N).to(torch.bfloat16).contiguous()
        if act == "gelu":
            d = d * saved
        elif act == "relu":
            d = torch.where(saved > 0, d, torch.zeros((), dtype=d.dtype, device=d.device))
        M, Kp = x2.shape
        dx = None
        if ctx.needs_input_grad[0]:
            if Kp % 64 == 0:
                dx = torch.empty(M, Kp, dtype=torch.bfloat16, device=d.device)
                tc_gemm(d.reshape(1, M, N), wb.reshape(1, N, Kp), dx.reshape(1, M, Kp), b_kn=True)
            else:
                dx = torch.mm(d, wb)
            dx = dx[:, :K].reshape(*lead, K)
        if _wgrad_ok(d, N, Kp):
            dw = tc_wgrad(d.reshape(1, M, N), x2.reshape(1, M, Kp), torch.zeros(1, N, Kp, device=d.device))[0]
        else:
            dw = torch.mm(d.t(), x2, out_dtype=torch.float32)
        dw = dw[:, :K].to(wdt)
        db = d.sum(0, dtype=torch.float32).to(bdt) if bdt is not None else None
        return dx, dw, db, None


def linear(lin: nn.Linear, x: torch.Tensor, act: str | None = None) -> torch.Tensor:
    """``act(lin(x))`` for act in {None, "gelu", "relu"}: on the tcgen05 GEMM
    when the shapes allow (bf16 input, output width a multiple of 64), else
    PyTorch."""
    if _gemm_ok(x) and x.dtype == torch.bfloat16 and lin.out_features % 64 == 0 and x.shape[-1] == lin.in_features:
        return _LinearNative.apply(x, lin.weight, lin.bias, act or "")
    y = lin(x)
    if act == "gelu":
        return F.gelu(y)
    if act == "relu":
        return F.relu(y)
    return y


def _rows_strided_ok(t: torch.Tensor) -> bool:
    """[B, L, N] bf16 view with contiguous rows and TMA-legal strides (a token
    range of a wider [B, T, N] buffer)."""
    return (t.dim() == 3 and t.stride(2) == 1 and t.stride(1) == t.shape[2] and (t.stride(0) * 2) % 16 == 0
            and t.data_ptr() % 16 == 0 and t.shape[1] % 64 == 0)


class _MLP2Native(torch.autograd.Function):
    """y = W2 GELU(W1 x + b1) + b2 (+ addend[l]) on the tcgen05 GEMM: the bias
    and GELU (with GELU' of the pre-activation stored for backward) fused into
    the first GEMM's epilogue, bias + per-position addend (the tokenizer's
    positional embedding) into the second's, the product with GELU' into the
    data-gradient GEMM. x [B, L, K]; addend [L, N] or None."""

    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2, addend):
        xb = x.contiguous().to(torch.bfloat16)
        B, L, K = xb.shape
        F_, N = w1.shape[0], w2.shape[0]
        w1b, w2b = w1.to(torch.bfloat16), w2.to(torch.bfloat16)
        rows = B * L
        v = lambda t: t.reshape(1, rows, t.shape[-1])  # noqa: E731
        r1 = b1.to(torch.bfloat16).reshape(1, 1, F_).expand(1, rows, F_)
        h = torch.empty(B, L, F_, dtype=torch.bfloat16, device=x.device)
        dact = torch.empty_like(h)                                # GELU'(pre-activation)
        tc_gemm(v(xb), w1b.reshape(1, F_, K), v(h), "gelu_d", R=r1, AUX=v(dact))
        add2 = b2.to(torch.bfloat16).reshape(1, N)
        if addend is not None:
            add2 = (addend.to(torch.float32) + b2.to(torch.float32)).to(torch.bfloat16)
            r2 = add2.reshape(1, L, N).expand(B, L, N)
        else:
            r2 = add2.reshape(1, 1, N).expand(B, L, N)
        out = torch.empty(B, L, N, dtype=torch.bfloat16, device=x.device)
        tc_gemm(v(h), w2b.reshape(1, N, F_), v(out), None, R=v(r2))
        ctx.save_for_backward(xb, h, dact, w1b, w2b)
        ctx.meta = (w1.dtype, b1.dtype, w2.dtype, b2.dtype, addend is not None,
                    addend.dtype if addend is not None else None)
        return out

    @staticmethod
    def backward(ctx, dout):
        xb, h, dact, w1b, w2b = ctx.saved_tensors
        dt_w1, dt_b1, dt_w2, dt_b2, has_add, dt_add = ctx.meta
        dout = dout.to(torch.bfloat16)
        B, L, N = dout.shape
        F_, K = w1b.shape
        rows = B * L
        v = lambda t: t.reshape(1, rows, t.shape[-1])  # noqa: E731
        # a tokenizer's output gradient arrives as a strided view (its token
        # range of the layer input's gradient): the GEMMs read it in place,
        # one batch per sample, instead of copying it
        strided = not dout.is_contiguous() and _rows_strided_ok(dout)
        if not strided:
            dout = dout.contiguous()
        d3 = dout if strided else v(dout)
        dpre = torch.empty(B, L, F_, dtype=torch.bfloat16, device=dout.device)
        tc_gemm(d3, w2b.reshape(1, N, F_), dpre if strided else v(dpre), "mul",
                R=dact if strided else v(dact), b_kn=True)
        dx = torch.empty(B, L, K, dtype=torch.bfloat16, device=dout.device)
        tc_gemm(v(dpre), w1b.reshape(1, F_, K), v(dx), b_kn=True)
        dp = dpre.reshape(rows, F_)
        if _wgrad_ok(dout, N, F_):
            dw2 = tc_wgrad(d3, h if strided else v(h), torch.zeros(1, N, F_, device=dout.device),
                           l_sum=strided)[0].to(dt_w2)
        else:
            dw2 = torch.mm(dout.reshape(rows, N).t(), h.reshape(rows, F_), out_dtype=torch.float32).to(dt_w2)
        if _wgrad_ok(dpre, F_, K):
            dw1 = tc_wgrad(v(dpre), v(xb), torch.zeros(1, F_, K, device=dout.device))[0].to(dt_w1)
        else:
            dw1 = torch.mm(dp.t(), xb.reshape(rows, K), out_dtype=torch.float32).to(dt_w1)
        dpos = dout.sum(0, dtype=torch.float32)         # [L, N], fp32 accumulation without an fp32 copy
        db2 = dpos.sum(0).to(dt_b2)
        db1 = dp.sum(0, dtype=torch.float32).to(dt_b1)
        return dx, dw1, db1, dw2, db2, (dpos.to(dt_add) if has_add else None)


class _PadCols(torch.autograd.Function):
    """w [N, K] -> [N, K + pad] with zero columns (gradient: the first K columns)."""

    @staticmethod
    def forward(ctx, w, pad: int):
        ctx.k = w.shape[1]
        return F.pad(w, (0, pad))

    @staticmethod
    def backward(ctx, g):
        return g[:, : ctx.k], None


def mlp2(x: torch.Tensor, l1: nn.Linear, l2: nn.Linear, addend: torch.Tensor | None = None) -> torch.Tensor:
    """l2(GELU(l1(x))) (+ addend[:L] broadcast over the batch).  On the
    tcgen05 GEMM when the shapes allow (bf16, K % 8, hidden / output % 64)."""
    if (x.dim() in (2, 3) and _gemm_ok(x) and x.dtype == torch.bfloat16 and l1.bias is not None
            and l2.bias is not None and l1.out_features % 64 == 0 and l2.out_features % 64 == 0
            and x.data_ptr() % 16 == 0):
        two_d = x.dim() == 2
        xin = x.unsqueeze(1) if two_d else x
        K = l1.in_features
        w1 = l1.weight
        if K % 64:  # pad the input features (and the weight's columns) to a multiple of 64: the
            # data gradient's GEMM then has an output width the tcgen05 kernel takes
            xin = F.pad(xin, (0, -K % 64))
            w1 = _PadCols.apply(w1, -K % 64)
        y = _MLP2Native.apply(xin, w1, l1.bias, l2.weight, l2.bias, addend)
        return y.squeeze(1) if two_d else y
    y = l2(F.gelu(l1(x)))
    if addend is not None:
        y = y + addend.to(y.dtype)
    return y

"""Pyramid causal attention.

Semantics (``primus_dlrm/models/onetrans.py:62-67,146-166``): queries are the
last ``q_len`` of ``kv_len`` tokens and attend causally with the mask aligned
bottom-right, ``kv_idx <= q_idx + (kv_len - q_len)``; scale ``1/sqrt(d)``.

Inputs are ``[B, L, H, d]`` views (any row stride, unit stride on ``d``);
the output is ``[B, q_len, H, d]`` contiguous.

Paths:
* ``native`` -- the sm_100a pyramid FMHA in ``_gemm`` when built and the
  shape is supported;
* ``sdpa`` -- ``F.scaled_dot_product_attention`` with a lower-right causal
  bias (flash / efficient backends);
* ``mask`` -- SDPA with an explicit boolean mask (reference ``sdpa`` path).
"""
from __future__ import annotations

import os

import torch
import torch.nn.functional as F

from primus_dlrm_b200.ops import _ext


def build_pyramid_mask(q_len: int, kv_len: int, device) -> torch.Tensor:
    """Boolean ``[q_len, kv_len]`` mask, True where attention is allowed."""
    off = kv_len - q_len
    qi = torch.arange(q_len, device=device).unsqueeze(1) + off
    ki = torch.arange(kv_len, device=device).unsqueeze(0)
    return ki <= qi


def _native_ok(q: torch.Tensor) -> bool:
    g = _ext.gemm() if (q.is_cuda and _ext.native_enabled(q.device)) else None
    return g is not None and hasattr(g, "fmha_fwd") and q.dtype == torch.bfloat16 and q.shape[-1] in (32, 64)


class _NativeFMHA(torch.autograd.Function):
    """q, k, v as separate [B, L, H, d] views (gradients returned separately)."""

    @staticmethod
    def forward(ctx, q, k, v, scale):
        G = _ext.gemm()
        o, lse = G.fmha_fwd(q, k, v, scale)
        ctx.scale = scale
        ctx.save_for_backward(q, k, v, o, lse)
        return o

    @staticmethod
    def backward(ctx, do):
        G = _ext.gemm()
        q, k, v, o, lse = ctx.saved_tensors
        B, ql, H, d = q.shape
        kl = k.shape[1]
        buf = torch.empty(B, kl, 3, H, d, dtype=q.dtype, device=q.device)
        G.fmha_bwd(q, k, v, o, lse, do.contiguous(), buf[:, :, 0], buf[:, :, 1], buf[:, :, 2], ctx.scale)
        return buf[:, kl - ql:, 0], buf[:, :, 1], buf[:, :, 2], None


# From this many queries the tcgen05 forward is faster on B200 (v6 pyramid,
# batch 2048: q 912 / kv 912 4.27 vs 4.52 ms, q 535 / kv 661 2.37 vs 2.44 ms;
# q 409 / kv 535 1.68 vs 1.66 ms and smaller layers favour the mma.sync kernel).
_TC_FWD_MIN_Q = int(os.environ.get("PD_ATTN_TC_FWD_MIN_Q", "500"))


def _tc_fwd_ok(qkv: torch.Tensor, q_len: int) -> bool:
    """The tcgen05 forward reads qkv through TMA maps: contiguous, d in {32, 64};
    used from _TC_FWD_MIN_Q queries up (PD_ATTN_TC_FWD=0: never, =1: always)."""
    g = _ext.gemm()
    mode = os.environ.get("PD_ATTN_TC_FWD", "")
    return (hasattr(g, "fmha_fwd_tc") and qkv.is_contiguous() and qkv.shape[-1] in (32, 64) and mode != "0"
            and (mode == "1" or q_len >= _TC_FWD_MIN_Q))


# Below this many queries the mma.sync backward is faster on B200 (v6 pyramid,
# batch 2048: q 32 / kv 158 0.56 vs 0.87 ms; q 158 / kv 283 1.86 vs 1.83 ms and
# every larger layer favour the tcgen05 kernel).
_TC_BWD_MIN_Q = int(os.environ.get("PD_ATTN_TC_BWD_MIN_Q", "100"))


def _tc_bwd_ok(qkv: torch.Tensor, q_len: int) -> bool:
    """tcgen05 backward: contiguous qkv, d = 32, q_len within its shared-memory
    dQ block and above the size where it beats the mma.sync backward."""
    g = _ext.gemm()
    return (hasattr(g, "fmha_bwd_tc") and qkv.is_contiguous() and qkv.shape[-1] == 32
            and _TC_BWD_MIN_Q <= q_len <= g.fmha_bwd_tc_max_q() and os.environ.get("PD_ATTN_TC_BWD", "1") != "0")


def _err_word(device) -> torch.Tensor:
    w = _ERR.get(device)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=device)
        _ERR[device] = w
    return w


_ERR: dict = {}
# calls of the native attention kernels (forward, backward) since import: a
# check that a run took the kernel path and not the PyTorch fallback
NATIVE_CALLS = {"fwd": 0, "bwd": 0}


def attention_error_code(device) -> int:
    """Error word of the tcgen05 attention kernels (0 = ok, 2 = a bounded wait ran out)."""
    w = _ERR.get(torch.device(device))
    return int(w.item()) if w is not None else 0


class _NativeFMHAFused(torch.autograd.Function):
    """Attention straight from the fused projection output qkv [B, T, 3, H, d]:
    queries are the last q_len rows; the gradient is one [B, T, 3, H, d]
    buffer written entirely by the backward kernels (no concatenation)."""

    @staticmethod
    def forward(ctx, qkv, q_len: int, scale: float):
        G = _ext.gemm()
        T = qkv.shape[1]
        q, k, v = qkv[:, T - q_len:, 0], qkv[:, :, 1], qkv[:, :, 2]
        if _tc_fwd_ok(qkv, q_len):
            o, lse = G.fmha_fwd_tc(qkv, q_len, scale, _err_word(qkv.device))
        else:
            o, lse = G.fmha_fwd(q, k, v, scale)
        NATIVE_CALLS["fwd"] += 1
        ctx.scale, ctx.q_len = scale, q_len
        ctx.save_for_backward(qkv, o, lse)
        return o

    @staticmethod
    def backward(ctx, do):
        G = _ext.gemm()
        qkv, o, lse = ctx.saved_tensors
        T, ql = qkv.shape[1], ctx.q_len
        dqkv = torch.empty_like(qkv)
        NATIVE_CALLS["bwd"] += 1
        if _tc_bwd_ok(qkv, ql):
            G.fmha_bwd_tc(qkv, o, lse, do.contiguous(), dqkv, ql, ctx.scale, _err_word(qkv.device))
            return dqkv, None, None
        G.fmha_bwd(qkv[:, T - ql:, 0], qkv[:, :, 1], qkv[:, :, 2], o, lse, do.contiguous(),
                   dqkv[:, :, 0], dqkv[:, :, 1], dqkv[:, :, 2], ctx.scale)
        return dqkv, None, None


def pyramid_attention_qkv(qkv: torch.Tensor, q_len: int) -> torch.Tensor:
    """qkv [B, T, 3, H, d] -> attention of the last q_len queries, [B, q_len, H, d]."""
    d = qkv.shape[-1]
    if _native_ok(qkv):
        return _NativeFMHAFused.apply(qkv, q_len, d ** -0.5)
    T = qkv.shape[1]
    return pyramid_attention(qkv[:, T - q_len:, 0], qkv[:, :, 1], qkv[:, :, 2], impl="mask")


def causal_attention_all_rows(qkv: torch.Tensor, n_heads: int) -> torch.Tensor:
    """Causal attention of every row of ``qkv`` [B, T, 3, H, d] -> [B, T, H, d].

    The pyramid keeps the LAST q_len queries, and the first kv_len - q_len rows
    of a causal score matrix are also its cheapest ones, so computing all rows
    (standard causal, q_len == kv_len) costs (kv-q)(kv-q+1)/2 extra pairs per
    head (~2% for the v6 pyramid) and runs every layer on the fast square
    causal kernels.  The caller keeps the last q_len rows.
    """
    q, k, v = qkv[:, :, 0].transpose(1, 2), qkv[:, :, 1].transpose(1, 2), qkv[:, :, 2].transpose(1, 2)
    out = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    return out.transpose(1, 2)


def pyramid_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, impl: str = "auto",
                      dropout_p: float = 0.0) -> torch.Tensor:
    """q [B, q_len, H, d]; k, v [B, kv_len, H, d] -> [B, q_len, H, d]."""
    B, ql, H, d = q.shape
    kl = k.shape[1]
    scale = d ** -0.5
    if impl in ("auto", "native") and dropout_p == 0.0 and _native_ok(q):
        return _NativeFMHA.apply(q, k, v, scale)
    qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    if impl == "mask" or not q.is_cuda:
        mask = build_pyramid_mask(ql, kl, q.device)
        out = F.scaled_dot_product_attention(qt, kt, vt, attn_mask=mask, dropout_p=dropout_p)
    else:
        from torch.nn.attention.bias import causal_lower_right
        out = F.scaled_dot_product_attention(qt, kt, vt, attn_mask=causal_lower_right(ql, kl),
                                             dropout_p=dropout_p)
    return out.transpose(1, 2).contiguous()

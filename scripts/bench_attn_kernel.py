#!/usr/bin/env python3
"""Standalone pyramid-attention benchmark over the layers of a OneTrans config
(the role of the reference's ``scripts/bench_attn_kernel.py``: per-layer
(q_len, kv_len) from ``compute_layer_shapes``, forward and backward timed
separately).

    python scripts/bench_attn_kernel.py --config configs/bench_onetrans_v6_b200.yaml
    python scripts/bench_attn_kernel.py --batch 256 --layers 1 --impl tc --pass fwd --reps 3

Implementations: ``mma`` (mma.sync kernels), ``tc`` (tcgen05 kernels), ``sdpa``
(PyTorch scaled_dot_product_attention with the bottom-right causal mask).
Times are CUDA-event device times after warm-up; TFLOPS count the causal
pairs only (4 d flops per pair forward, 8 d backward).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402


def layer_shapes(config) -> list[tuple[int, int]]:
    from primus_dlrm_b200.models.onetrans import pyramid_schedule
    ot = config.model.transformer
    L_S = config.sequence_length_total()
    sched = pyramid_schedule(L_S, ot.n_ns_tokens, ot.n_layers) if ot.use_pyramid else [L_S] * ot.n_layers
    shapes, kv = [], L_S + ot.n_ns_tokens
    for l in range(ot.n_layers):
        q = sched[l] + ot.n_ns_tokens
        shapes.append((q, kv))
        kv = q
    return shapes


def _time(fn, reps: int) -> float:
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(reps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / reps


def main(argv=None) -> dict:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--config", default=str(ROOT / "configs" / "bench_onetrans_v6_b200.yaml"))
    p.add_argument("--batch", type=int, default=2048)
    p.add_argument("--impl", default="all", choices=["all", "mma", "tc", "sdpa"])
    p.add_argument("--pass", dest="which", default="both", choices=["both", "fwd", "bwd"])
    p.add_argument("--layers", default="", help="comma-separated layer indices (default: all)")
    p.add_argument("--reps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--json", action="store_true")
    args = p.parse_args(argv)

    from primus_dlrm_b200.config import Config
    from primus_dlrm_b200.ops import _ext
    from primus_dlrm_b200.ops.attention import build_pyramid_mask
    cfg = Config.load(args.config)
    ot = cfg.model.transformer
    H, d = ot.n_heads, ot.d_model // ot.n_heads
    shapes = layer_shapes(cfg)
    pick = [int(x) for x in args.layers.split(",") if x.strip()] or list(range(len(shapes)))
    G = _ext.gemm()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    impls = ["mma", "tc", "sdpa"] if args.impl == "all" else [args.impl]
    scale = d ** -0.5
    rows, totals = [], {}
    for li in pick:
        ql, kl = shapes[li]
        B = args.batch
        qkv = torch.randn(B, kl, 3, H, d, device="cuda").to(torch.bfloat16)
        q, k, v = qkv[:, kl - ql:, 0], qkv[:, :, 1], qkv[:, :, 2]
        do = torch.randn(B, ql, H, d, device="cuda").to(torch.bfloat16)
        dqkv = torch.empty_like(qkv)
        pairs = ql * kl - ql * (ql - 1) / 2
        row = {"layer": li, "q_len": ql, "kv_len": kl}
        for impl in impls:
            if impl == "tc" and d != 32 and args.which != "fwd":
                continue
            if impl == "sdpa":
                mask = build_pyramid_mask(ql, kl, qkv.device)
                qt = q.transpose(1, 2).detach().requires_grad_(True)
                kt = k.transpose(1, 2).detach().requires_grad_(True)
                vt = v.transpose(1, 2).detach().requires_grad_(True)
                fwd = lambda: torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, attn_mask=mask)  # noqa: E731
                out = fwd()
                gout = do.transpose(1, 2)
                bwd = lambda: torch.autograd.grad(out, (qt, kt, vt), gout, retain_graph=True)  # noqa: E731
            elif impl == "mma":
                fwd = lambda: G.fmha_fwd(q, k, v, scale)  # noqa: E731
                o, lse = fwd()
                bwd = lambda: G.fmha_bwd(q, k, v, o, lse, do, dqkv[:, :, 0], dqkv[:, :, 1], dqkv[:, :, 2], scale)  # noqa: E731
            else:
                fwd = lambda: G.fmha_fwd_tc(qkv, ql, scale, err)  # noqa: E731
                o, lse = G.fmha_fwd(q, k, v, scale)
                bwd = lambda: G.fmha_bwd_tc(qkv, o, lse, do, dqkv, ql, scale, err)  # noqa: E731
            for which, fn, flop in (("fwd", fwd, 4), ("bwd", bwd, 8)):
                if args.which not in ("both", which):
                    continue
                for _ in range(args.warmup):
                    fn()
                ms = _time(fn, args.reps)
                row[f"{impl}_{which}_ms"] = round(ms, 4)
                row[f"{impl}_{which}_tflops"] = round(flop * B * H * d * pairs / ms / 1e9, 1)
                totals[f"{impl}_{which}_ms"] = totals.get(f"{impl}_{which}_ms", 0.0) + ms
        rows.append(row)
        if not args.json:
            print("  ".join(f"{k}={v}" for k, v in row.items()), flush=True)
    if int(err.item()) != 0:
        raise RuntimeError(f"attention kernel error word {int(err.item())}")
    res = {"batch": args.batch, "heads": H, "head_dim": d, "layers": rows,
           "totals_ms": {k: round(v, 3) for k, v in totals.items()}}
    print(json.dumps(res) if args.json else "totals: " + json.dumps(res["totals_ms"]))
    return res


if __name__ == "__main__":
    main()

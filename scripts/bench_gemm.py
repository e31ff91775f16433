#!/usr/bin/env python3
"""Micro-benchmark of the tcgen05 GEMM (``_gemm.tc_gemm``) on the projection
shapes of a OneTrans layer, against cuBLAS (``torch.matmul``) on the same
operands, with roofline fractions of the measured copy bandwidth and bf16
GEMM rate (``MEASURED_PEAKS.json`` at the repo root, when present).

    python scripts/bench_gemm.py                      # layer-0 shapes at batch 2048
    python scripts/bench_gemm.py --rows 233472 --reps 20

Shapes (rows = batch x tokens):
  qkv        [rows, 256]  x [768, 256]^T               plain
  ffn_up     [rows, 256]  x [1024, 256]^T  GELU, GELU' stored (AUX)  (training forward)
  ffn_down   [rows, 1024] x [256, 1024]^T  + residual
  ffn_dgrad  [rows, 256]  x [1024, 256]^T  x stored GELU'           (training backward)
  gelu_pre   as ffn_up, storing the pre-activation instead
  dgelu_pre  as ffn_dgrad, GELU' recomputed from the pre-activation
Times are CUDA-event device times per call after warm-up; each call's
inputs exceed L2 at the default size.  Bytes count A + B + C (+ R / AUX).

With ``--wgrad`` the weight-gradient products of the same layer (dW = dY^T X
over all rows, and the per-NS-token ones over the batch) are timed instead:
the tcgen05 split-K kernel (``tc_wgrad``) against cuBLAS with fp32 output.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402


def _time(fn, reps: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(reps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / reps


def main(argv=None) -> list[dict]:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--rows", type=int, default=2048 * 912)
    p.add_argument("--reps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--shapes", default="qkv,ffn_up,ffn_down,ffn_dgrad")
    p.add_argument("--wgrad", action="store_true")
    a = p.parse_args(argv)
    if a.wgrad:
        return _wgrad(a)
    from primus_dlrm_b200.ops.dense import tc_gemm
    peaks = {}
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    hbm = float(peaks.get("hbm_gbs", 6650.0)) * 1e9
    flops_peak = float(peaks.get("bf16_tflops", 1590.0)) * 1e12
    dev = torch.device("cuda")
    M = a.rows
    bf = dict(dtype=torch.bfloat16, device=dev)
    specs = {
        "qkv": (256, 768, None),
        "ffn_up": (256, 1024, "gelu_d"),
        "ffn_down": (1024, 256, "residual"),
        "ffn_dgrad": (256, 1024, "mul"),
        "gelu_pre": (256, 1024, "gelu"),
        "dgelu_pre": (256, 1024, "dgelu"),
    }
    out = []
    for name in [s.strip() for s in a.shapes.split(",") if s.strip()]:
        K, N, epi = specs[name]
        A = torch.randn(1, M, K, **bf)
        B = torch.randn(1, N, K, **bf) * 0.05
        C = torch.empty(1, M, N, **bf)
        R = torch.randn(1, M, N, **bf) if epi in ("residual", "dgelu", "mul") else None
        X = torch.empty(1, M, N, **bf) if epi in ("gelu", "gelu_d") else None
        ms = _time(lambda: tc_gemm(A, B, C, epi, R=R, AUX=X), a.reps, a.warmup)
        ref_ms = _time(lambda: torch.matmul(A[0], B[0].t()), a.reps, a.warmup)
        flops = 2.0 * M * N * K
        nbytes = 2.0 * (M * K + N * K + M * N * (1 + (R is not None) + (X is not None)))
        roof_ms = max(flops / flops_peak, nbytes / hbm) * 1e3
        row = {"shape": name, "M": M, "N": N, "K": K, "epi": epi or "none", "ms": round(ms, 4),
               "tflops": round(flops / ms / 1e9, 1), "gbs": round(nbytes / ms / 1e6, 1),
               "roofline_ms": round(roof_ms, 4), "frac_of_roofline": round(roof_ms / ms, 3),
               "cublas_plain_ms": round(ref_ms, 4)}
        out.append(row)
        print(json.dumps(row), flush=True)
    return out


def _wgrad(a) -> list[dict]:
    from primus_dlrm_b200.ops.dense import tc_wgrad
    peaks = {}
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    hbm = float(peaks.get("hbm_gbs", 6650.0)) * 1e9
    dev = torch.device("cuda")
    rows, out = a.rows, []
    for name, M, N in (("qkv", 768, 256), ("ffn_up", 1024, 256), ("ffn_down", 256, 1024), ("out_proj", 256, 256)):
        A = torch.randn(1, rows, M, device=dev).to(torch.bfloat16)
        B = torch.randn(1, rows, N, device=dev).to(torch.bfloat16)
        C = torch.zeros(1, M, N, device=dev)
        ms = _time(lambda: tc_wgrad(A, B, C), a.reps, a.warmup)
        ref_ms = _time(lambda: torch.mm(A[0].t(), B[0], out_dtype=torch.float32), a.reps, a.warmup)
        nbytes = 2.0 * rows * (M + N)
        row = {"dW": name, "M": M, "N": N, "rows": rows, "tc_ms": round(ms, 4), "cublas_ms": round(ref_ms, 4),
               "tc_tflops": round(2.0 * rows * M * N / ms / 1e9, 1), "hbm_roofline_ms": round(nbytes / hbm * 1e3, 4)}
        out.append(row)
        print(json.dumps(row), flush=True)
    return out


if __name__ == "__main__":
    main()

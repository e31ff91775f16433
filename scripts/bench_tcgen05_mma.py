#!/usr/bin/env python3
"""Issue / execution rate of back-to-back ``tcgen05.mma`` instructions
(M = 128, K = 16, bf16 -> fp32) for the operand forms the attention and GEMM
kernels use, one CTA per SM (``_gemm.tc_mma_rate``).

    python scripts/bench_tcgen05_mma.py                # the default table
    python scripts/bench_tcgen05_mma.py --iters 4096 --json

Each row gives the median over SMs of cycles per instruction (execution:
first issue to commit completion) and of issue cycles per instruction, and
the tensor rate this implies per SM (dense bf16 FLOP per cycle; 8192 is the
nominal 2.25 PFLOP/s over 148 SMs at 1.86 GHz).
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

MODES = {0: "SS A:K B:K", 1: "SS A:K B:MN", 2: "SS A:MN B:MN", 3: "TS B:K", 4: "TS B:MN"}

ISSUE = {0: "lone lane", 1: "warp+elect", 2: "warp+elect+mask"}

DEFAULT_CASES = [
    # (mode, n, nacc, swz)
    (0, 256, 1, 2), (0, 128, 1, 2), (0, 64, 1, 2), (0, 32, 1, 2), (0, 16, 1, 2),
    (0, 128, 1, 4), (0, 32, 1, 4), (0, 32, 3, 4),
    (1, 32, 1, 4), (1, 32, 3, 4), (1, 64, 1, 2),
    (2, 32, 1, 4), (2, 32, 3, 2),
    (3, 256, 1, 2), (3, 128, 1, 2), (3, 64, 1, 2), (3, 32, 1, 2), (3, 32, 3, 2),
    (4, 32, 1, 4), (4, 32, 3, 4), (4, 64, 1, 2),
]


def run(cases, iters: int, issues=(0, 1, 2)) -> list[dict]:
    import torch

    from primus_dlrm_b200.ops import _ext

    g = _ext.gemm()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rows = []
    for (mode, n, nacc, swz), issue in [(c, i) for i in issues for c in cases]:
        g.tc_mma_rate(mode, n, 64, nacc, swz, issue, err)  # warm-up
        out = g.tc_mma_rate(mode, n, iters, nacc, swz, issue, err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0, f"probe wait timed out (mode {mode}, n {n})"
        issue_cyc = out[:, 0].double().median().item() / iters
        total = out[:, 1].double().median().item() / iters
        flop = 2.0 * 128 * n * 16
        rows.append({"issue": ISSUE[issue], "mode": MODES[mode], "n": n, "nacc": nacc,
                     "swizzle_bytes": 128 if swz == 2 else 64,
                     "cycles_per_mma": round(total, 2), "issue_cycles_per_mma": round(issue_cyc, 2),
                     "flop_per_cycle_per_sm": round(flop / total, 1)})
    return rows


VARS = {0: "fixed operands", 1: "B advances", 2: "A advances", 3: "runtime acc flag", 4: "not unrolled",
        5: "k-loop (1+2+3)", 10: "A:K128 B:K128", 11: "A:K128 B:MN64", 12: "A:MN128 B:MN64", 13: "A:K64 B:K64"}


def run_vars(iters: int) -> list[dict]:
    """Single and four issuers with operands that change per instruction the
    way a k-loop changes them."""
    import torch

    from primus_dlrm_b200.ops import _ext

    g = _ext.gemm()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rows = []
    for ts in (1, 0):
        for n in (32, 128):
            for var in (10, 11, 12, 13):
                if ts and var == 12:
                    continue                     # A from TMEM has no MN-major form
                for issuers in (1, 4):
                    g.tc_mma_burst(n, 4, issuers, 1, ts, 1, 1, var, err)
                    out = g.tc_mma_burst(n, iters, issuers, 1, ts, 1, 1, var, err)
                    torch.cuda.synchronize()
                    assert int(err.item()) == 0, "probe wait timed out"
                    cyc = out[:, 1:2 * issuers:2].max(dim=1).values.double().median().item() / (iters * 16)
                    rows.append({"operands": "TS" if ts else "SS", "n": n, "variant": VARS[var], "issuers": issuers,
                                 "cycles_per_mma_per_issuer": round(cyc, 2),
                                 "flop_per_cycle_per_sm": round(issuers / cyc * 2.0 * 128 * n * 16, 1)})
    return rows


def run_burst(iters: int) -> list[dict]:
    """Unrolled issue (16 MMAs of straight-line code per loop trip); 1 or 2
    issuing warps per CTA, 1 or 2 CTAs per SM."""
    import torch

    from primus_dlrm_b200.ops import _ext

    g = _ext.gemm()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rows = []
    for ts in (0, 1):
        for n in (32, 64, 128, 256):
            for issuers, per_sm, ws, lanes in ((1, 1, 1, 1), (2, 1, 1, 1), (1, 2, 1, 1), (4, 1, 1, 1), (2, 1, 4, 1),
                                               (4, 1, 4, 1), (1, 1, 1, 2), (1, 1, 1, 4), (2, 1, 1, 2)):
                if lanes * issuers * n > 448 and n <= 32:
                    continue
                g.tc_mma_burst(n, 4, issuers, per_sm, ts, ws, lanes, 0, err)
                out = g.tc_mma_burst(n, iters, issuers, per_sm, ts, ws, lanes, 0, err)
                torch.cuda.synchronize()
                assert int(err.item()) == 0, "probe wait timed out"
                per_warp = out[:, 1:2 * issuers:2].max(dim=1).values.double()
                cyc = per_warp.median().item() / (iters * 16)          # cycles per MMA of one issuer
                sm_mmas_per_cycle = issuers * per_sm * lanes / cyc
                rows.append({"operands": "TS" if ts else "SS", "n": n, "issuers_per_cta": issuers,
                             "same_subpartition": ws == 4, "lanes_per_warp": lanes,
                             "ctas_per_sm": per_sm, "cycles_per_mma_per_issuer": round(cyc, 2),
                             "flop_per_cycle_per_sm": round(sm_mmas_per_cycle * 2.0 * 128 * n * 16, 1)})
    return rows


def main(argv=None) -> list[dict]:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--iters", type=int, default=2048)
    p.add_argument("--issue", default="0,1,2", help="issue styles: 0 lone lane, 1 warp + elect.sync, "
                   "2 as 1 with the lane-mask operand form")
    p.add_argument("--burst", action="store_true", help="unrolled issue, several issuers per SM")
    p.add_argument("--vars", action="store_true", help="operands that change per instruction (k-loop forms)")
    p.add_argument("--json", action="store_true")
    a = p.parse_args(argv)
    if a.vars:
        rows = run_vars(max(a.iters // 16, 1))
        if a.json:
            print(json.dumps(rows))
        else:
            print(f"{'ops':4s} {'N':>4s} {'variant':18s} {'iss':>3s} {'cyc/mma/issuer':>15s} {'FLOP/cyc/SM':>12s}")
            for r in rows:
                print(f"{r['operands']:4s} {r['n']:4d} {r['variant']:18s} {r['issuers']:3d} "
                      f"{r['cycles_per_mma_per_issuer']:15.2f} {r['flop_per_cycle_per_sm']:12.1f}")
        return rows
    if a.burst:
        rows = run_burst(max(a.iters // 16, 1))
        if a.json:
            print(json.dumps(rows))
        else:
            print(f"{'ops':4s} {'N':>4s} {'iss':>3s} {'sameSP':>6s} {'lanes':>5s} {'cta/SM':>6s} {'cyc/mma/issuer':>15s} "
                  f"{'FLOP/cyc/SM':>12s}")
            for r in rows:
                print(f"{r['operands']:4s} {r['n']:4d} {r['issuers_per_cta']:3d} {int(r['same_subpartition']):6d} "
                      f"{r['lanes_per_warp']:5d} "
                      f"{r['ctas_per_sm']:6d} "
                      f"{r['cycles_per_mma_per_issuer']:15.2f} {r['flop_per_cycle_per_sm']:12.1f}")
        return rows
    rows = run(DEFAULT_CASES, a.iters, tuple(int(x) for x in a.issue.split(",")))
    if a.json:
        print(json.dumps(rows))
    else:
        print(f"{'issue':16s} {'operands':14s} {'N':>4s} {'acc':>3s} {'swz':>4s} {'cyc/mma':>8s} {'issue':>6s} "
              f"{'FLOP/cyc/SM':>12s}")
        for r in rows:
            print(f"{r['issue']:16s} {r['mode']:14s} {r['n']:4d} {r['nacc']:3d} {r['swizzle_bytes']:4d} "
                  f"{r['cycles_per_mma']:8.2f} {r['issue_cycles_per_mma']:6.2f} {r['flop_per_cycle_per_sm']:12.1f}")
    return rows


if __name__ == "__main__":
    main()

"""Offline analysis of the Chrome traces written by ``training.tracer``
(the reference's ``scripts/analyze_comms.py``, ``analyze_gemm_trace.py`` and
``stitch_traces.py``):

* ``kernel_breakdown`` -- device time per kernel category (GEMM, attention,
  embedding, norm, loss / optimizer, communication, elementwise, other), the
  table of the reference's perf analysis;
* ``comm_report`` -- collective kernels with algorithm / bus bandwidth
  (nccl-tests factors: all-reduce 2(n-1)/n, all-gather / reduce-scatter /
  all-to-all (n-1)/n) and the exposed part of communication: time not
  covered by the union of compute-kernel intervals on the same device;
* ``gemm_report`` -- (M, N, K) of GEMM kernels from the CPU op that launched
  them (matched by the trace's correlation / External id) and achieved TF/s;
* ``idle_gaps`` -- stretches where a device runs no kernel at all, with the
  host op that was running when each began (launch-bound or host-synchronised
  regions of a step);
* ``stitch`` -- merge per-rank traces into one file with per-rank process ids.

CLI: ``python -m primus_dlrm_b200.training.trace_analysis {breakdown,comms,gemm,gaps,stitch} ...``
"""
from __future__ import annotations

import argparse
import gzip
import json
import re
from collections import defaultdict
from pathlib import Path

CATEGORIES = (
    ("communication", re.compile(r"nccl|all_?reduce|all_?gather|reduce_?scatter|alltoall|sendrecv|"
                                 r"push_rows|signal_barrier|owner_keys", re.I)),
    ("attention", re.compile(r"fmha|flash|attention|sdpa|fwd_sm100|bwd_sm100", re.I)),
    ("embedding", re.compile(r"gather_kernel|pooled_kernel|keys_kernel|reduce_update|embedding|tbe|"
                             r"radixsort|segment", re.I)),
    ("gemm", re.compile(r"gemm|nvjet|cutlass|cublas|sgemm|hgemm|splitkreduce", re.I)),
    ("norm", re.compile(r"norm", re.I)),
    ("loss_optimizer", re.compile(r"heads_loss|adamw|sqnorm|multi_tensor|optim|loss", re.I)),
    ("elementwise", re.compile(r"elementwise|vectorized|unrolled|copy|fill|cat|reduce_kernel|memset|memcpy",
                               re.I)),
)


def load_trace(path: str | Path) -> dict:
    p = Path(path)
    opener = gzip.open if p.suffix == ".gz" else open
    with opener(p, "rt") as f:
        return json.load(f)


def _events(trace: dict) -> list[dict]:
    return trace.get("traceEvents", trace if isinstance(trace, list) else [])


def _is_kernel(e: dict) -> bool:
    return e.get("ph") == "X" and str(e.get("cat", "")).lower() in ("kernel", "gpu_memcpy", "gpu_memset")


def categorize(name: str) -> str:
    for cat, rx in CATEGORIES:
        if rx.search(name):
            return cat
    return "other"


def _merge(intervals: list[tuple[float, float]]) -> list[tuple[float, float]]:
    out: list[list[float]] = []
    for a, b in sorted(intervals):
        if out and a <= out[-1][1]:
            out[-1][1] = max(out[-1][1], b)
        else:
            out.append([a, b])
    return [(a, b) for a, b in out]


def _overlap(a: float, b: float, merged: list[tuple[float, float]]) -> float:
    tot = 0.0
    for x, y in merged:
        if y <= a:
            continue
        if x >= b:
            break
        tot += min(b, y) - max(a, x)
    return tot


def kernel_breakdown(trace: dict, steps: int = 1) -> dict:
    """{category: ms per step} over all device kernels (summed over devices)."""
    tot = defaultdict(float)
    for e in _events(trace):
        if _is_kernel(e):
            tot[categorize(e.get("name", ""))] += float(e.get("dur", 0.0))
    all_us = sum(tot.values()) or 1.0
    return {c: {"ms_per_step": v / 1000.0 / max(steps, 1), "share": v / all_us}
            for c, v in sorted(tot.items(), key=lambda kv: -kv[1])}


_BUS = {"all_reduce": lambda n: 2.0 * (n - 1) / n, "all_gather": lambda n: (n - 1) / n,
        "reduce_scatter": lambda n: (n - 1) / n, "all_to_all": lambda n: (n - 1) / n,
        "broadcast": lambda n: 1.0, "send_recv": lambda n: 1.0}
_DTYPE_BYTES = {"float": 4, "float32": 4, "bfloat16": 2, "half": 2, "float16": 2, "long": 8, "int64": 8,
                "int": 4, "int32": 4, "byte": 1, "uint8": 1}


def _coll_kind(name: str) -> str:
    n = name.lower()
    for k, rx in (("all_reduce", r"allreduce|all_reduce"), ("all_gather", r"allgather|all_gather"),
                  ("reduce_scatter", r"reducescatter|reduce_scatter"), ("all_to_all", r"alltoall|all_to_all"),
                  ("broadcast", r"broadcast"), ("send_recv", r"sendrecv|send|recv")):
        if re.search(rx, n):
            return k
    return "other"


def comm_report(trace: dict, world_size: int = 0) -> dict:
    """Collectives with bandwidths and the exposed communication time."""
    ev = _events(trace)
    # message sizes from the c10d CPU records (record_param_comms), by External id
    sizes = {}
    for e in ev:
        a = e.get("args", {}) or {}
        if "In msg nelems" in a or "Out msg nelems" in a:
            nel = max(int(a.get("In msg nelems", 0) or 0), int(a.get("Out msg nelems", 0) or 0))
            nbytes = nel * _DTYPE_BYTES.get(str(a.get("dtype", "float")).lower(), 4)
            ext = a.get("External id")
            if ext is not None:
                sizes[ext] = (nbytes, int(a.get("Group size", world_size) or world_size))
    by_dev: dict = defaultdict(lambda: {"comm": [], "compute": []})
    for e in ev:
        if not _is_kernel(e):
            continue
        dev = (e.get("pid"), (e.get("args", {}) or {}).get("device"))
        iv = (float(e["ts"]), float(e["ts"]) + float(e.get("dur", 0.0)))
        if categorize(e.get("name", "")) == "communication":
            by_dev[dev]["comm"].append((iv, e))
        else:
            by_dev[dev]["compute"].append(iv)
    colls = defaultdict(lambda: {"count": 0, "ms": 0.0, "bytes": 0, "exposed_ms": 0.0, "algbw": [], "busbw": []})
    total_ms = exposed_ms = 0.0
    for dev, d in by_dev.items():
        merged = _merge(d["compute"])
        for (a, b), e in d["comm"]:
            dur = b - a
            exp = dur - _overlap(a, b, merged)
            kind = _coll_kind(e.get("name", ""))
            c = colls[kind]
            c["count"] += 1
            c["ms"] += dur / 1000.0
            c["exposed_ms"] += exp / 1000.0
            total_ms += dur / 1000.0
            exposed_ms += exp / 1000.0
            ext = (e.get("args", {}) or {}).get("External id")
            if ext in sizes and dur > 0:
                nbytes, n = sizes[ext]
                c["bytes"] += nbytes
                alg = nbytes / (dur * 1e-6) / 1e9
                c["algbw"].append(alg)
                if n > 1 and kind in _BUS:
                    c["busbw"].append(alg * _BUS[kind](n))
    out = {}
    for k, c in colls.items():
        out[k] = {"count": c["count"], "ms": round(c["ms"], 3), "exposed_ms": round(c["exposed_ms"], 3),
                  "bytes": c["bytes"],
                  "algbw_gbs": round(sum(c["algbw"]) / len(c["algbw"]), 1) if c["algbw"] else None,
                  "busbw_gbs": round(sum(c["busbw"]) / len(c["busbw"]), 1) if c["busbw"] else None}
    return {"collectives": out, "total_ms": round(total_ms, 3), "exposed_ms": round(exposed_ms, 3),
            "overlapped_ms": round(total_ms - exposed_ms, 3)}


_MM_OPS = ("aten::mm", "aten::addmm", "aten::bmm", "aten::matmul", "aten::linear", "aten::baddbmm")


def _mnk(op: str, dims: list) -> tuple[int, int, int, int] | None:
    try:
        if op in ("aten::mm", "aten::matmul") and len(dims) >= 2 and len(dims[0]) == 2:
            (m, k), (_, n) = dims[0], dims[1]
            return 1, m, n, k
        if op == "aten::addmm":
            (m, k), (_, n) = dims[1], dims[2]
            return 1, m, n, k
        if op in ("aten::bmm", "aten::baddbmm"):
            a, b = (dims[0], dims[1]) if op == "aten::bmm" else (dims[1], dims[2])
            return a[0], a[1], b[2], a[2]
        if op == "aten::linear":
            x, w = dims[0], dims[1]
            m = 1
            for s in x[:-1]:
                m *= s
            return 1, m, w[0], w[1]
    except (IndexError, TypeError, ValueError):
        return None
    return None


def gemm_report(trace: dict, top: int = 30) -> list[dict]:
    """(batch, M, N, K), count, time and TF/s per GEMM shape."""
    ev = _events(trace)
    shape_of = {}
    for e in ev:
        if e.get("ph") == "X" and e.get("name") in _MM_OPS:
            a = e.get("args", {}) or {}
            s = _mnk(e["name"], a.get("Input Dims", []))
            if s is not None:
                shape_of[a.get("External id")] = s
    agg = defaultdict(lambda: {"count": 0, "us": 0.0})
    for e in ev:
        if _is_kernel(e) and categorize(e.get("name", "")) == "gemm":
            s = shape_of.get((e.get("args", {}) or {}).get("External id"))
            if s is None:
                continue
            agg[s]["count"] += 1
            agg[s]["us"] += float(e.get("dur", 0.0))
    rows = []
    for (bt, m, n, k), v in agg.items():
        flops = 2.0 * bt * m * n * k * v["count"]
        rows.append({"batch": bt, "M": m, "N": n, "K": k, "count": v["count"], "ms": round(v["us"] / 1000, 3),
                     "tflops": round(flops / (v["us"] * 1e-6) / 1e12, 1) if v["us"] > 0 else None})
    return sorted(rows, key=lambda r: -r["ms"])[:top]


def stitch(paths: list[str | Path], out: str | Path) -> Path:
    """Merge per-rank traces: rank r's process ids become r * 10^6 + pid,
    each labelled ``rank r / <original name>``."""
    merged = []
    for r, p in enumerate(paths):
        names = {}
        for e in _events(load_trace(p)):
            e = dict(e)
            pid = e.get("pid", 0)
            try:
                new_pid = r * 1_000_000 + int(pid)
            except (TypeError, ValueError):
                new_pid = r * 1_000_000 + (abs(hash(pid)) % 100_000)
            if e.get("ph") == "M" and e.get("name") == "process_name":
                names[new_pid] = True
                e["args"] = {"name": f"rank {r} / {(e.get('args') or {}).get('name', pid)}"}
            e["pid"] = new_pid
            merged.append(e)
        for pid in {e["pid"] for e in merged if e["pid"] // 1_000_000 == r} - set(names):
            merged.append({"ph": "M", "name": "process_name", "pid": pid, "args": {"name": f"rank {r}"}})
    out = Path(out)
    with open(out, "w") as f:
        json.dump({"traceEvents": merged}, f)
    return out


def idle_gaps(trace: dict, min_us: float = 20.0, top: int = 30) -> dict:
    """Device idle gaps (no kernel, copy or memset on any stream) longer than
    ``min_us``, per device, with the innermost host op running at each gap's
    start.  Totals cover the span from the first to the last device event."""
    ev = _events(trace)
    by_dev: dict = defaultdict(list)
    for e in ev:
        if _is_kernel(e):
            dev = (e.get("args") or {}).get("device", e.get("pid"))
            by_dev[dev].append((float(e["ts"]), float(e["ts"]) + float(e.get("dur", 0.0))))
    host = sorted((float(e["ts"]), float(e["ts"]) + float(e.get("dur", 0.0)), e.get("name", ""))
                  for e in ev if e.get("ph") == "X" and str(e.get("cat", "")).lower() in ("cpu_op", "user_annotation"))

    def host_op(t: float) -> str:
        best, best_len = "", float("inf")
        for a, b, n in host:          # innermost op that contains t
            if a > t:
                break
            if b >= t and b - a < best_len:
                best, best_len = n, b - a
        return best

    out = {}
    for dev, iv in by_dev.items():
        m = _merge(iv)
        gaps = [(m[i][1], m[i + 1][0]) for i in range(len(m) - 1) if m[i + 1][0] - m[i][1] >= min_us]
        span = m[-1][1] - m[0][0] if m else 0.0
        idle = sum(b - a for a, b in gaps)
        rows = sorted(gaps, key=lambda g: g[0] - g[1])[:top]
        out[str(dev)] = {
            "span_ms": round(span / 1000, 3), "idle_ms": round(idle / 1000, 3), "n_gaps": len(gaps),
            "top": [{"start_us": round(a - m[0][0], 1), "gap_us": round(b - a, 1), "host_op": host_op(a)}
                    for a, b in rows],
        }
    return out


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="Analyse torch.profiler Chrome traces")
    sub = p.add_subparsers(dest="cmd", required=True)
    b = sub.add_parser("breakdown"); b.add_argument("trace"); b.add_argument("--steps", type=int, default=1)
    c = sub.add_parser("comms"); c.add_argument("trace"); c.add_argument("--world-size", type=int, default=0)
    g = sub.add_parser("gemm"); g.add_argument("trace"); g.add_argument("--top", type=int, default=30)
    i = sub.add_parser("gaps"); i.add_argument("trace"); i.add_argument("--min-us", type=float, default=20.0)
    s = sub.add_parser("stitch"); s.add_argument("traces", nargs="+"); s.add_argument("--out", required=True)
    a = p.parse_args(argv)
    if a.cmd == "breakdown":
        res = kernel_breakdown(load_trace(a.trace), a.steps)
    elif a.cmd == "comms":
        res = comm_report(load_trace(a.trace), a.world_size)
    elif a.cmd == "gemm":
        res = gemm_report(load_trace(a.trace), a.top)
    elif a.cmd == "gaps":
        res = idle_gaps(load_trace(a.trace), a.min_us)
    else:
        res = str(stitch(a.traces, a.out))
    print(json.dumps(res, indent=1))


if __name__ == "__main__":
    main()

#!/usr/bin/env python3
"""Embedding lookup + exchange micro-benchmark (the lookup / all-to-all sweep
of the embedding micro-benchmark config): one table sharded over the ranks,
``--ids`` ids per sample (sequence lookup) or pooled bags of ``--pooling``
ids, Zipf-distributed ids. Forward (lookup + exchange into the consumer's
activation buffer) and backward (gradient exchange + fused sparse optimizer)
are timed separately with CUDA events, max over ranks, for the peer-memory
executor (``--comm peer``) and the NCCL all-to-all baseline (``--comm nccl``).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 scripts/bench_embedding.py \\
        --rows 9400000 --dim 128 --ids 912 --batch 2048 --comm peer
    ... --pooling 64 --ids 64          # pooled (mean) bags

The roofline is the time to move the remote share of the bytes over NVLink
at ``--link-gbs`` (770 GB/s per direction measured on this pool): forward
rows read from other ranks, backward deduplicated gradient rows written to
their owners.
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
import torch.distributed as dist  # noqa: E402


def main(argv=None) -> dict:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--rows", type=int, default=9_400_000)
    p.add_argument("--dim", type=int, default=128)
    p.add_argument("--ids", type=int, default=912, help="ids per sample")
    p.add_argument("--pooling", type=int, default=0, help="> 0: mean-pooled bags of this many ids")
    p.add_argument("--batch", type=int, default=2048, help="samples per rank")
    p.add_argument("--zipf", type=float, default=1.05)
    p.add_argument("--sharding", default="row_wise", choices=["row_wise", "table_wise"])
    p.add_argument("--comm", default="peer", choices=["peer", "nccl"])
    p.add_argument("--optimizer", default="adam", choices=["sgd", "adagrad", "row_wise_adagrad", "adam"])
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--link-gbs", type=float, default=770.0)
    a = p.parse_args(argv)

    from primus_dlrm_b200.config import EmbeddingTableConfig
    from primus_dlrm_b200.data.synthetic import zipf_ids
    from primus_dlrm_b200.models.embedding import Embeddings
    from primus_dlrm_b200.ops.embedding import SparseOptimizer
    from primus_dlrm_b200.parallel.planner import TablePlan
    from primus_dlrm_b200.parallel.setup import get_local_rank, get_rank, get_world_size, init_distributed
    from primus_dlrm_b200.parallel.sharded_embedding import shard_embeddings

    init_distributed(timeout_s=300)
    rank, world = get_rank(), get_world_size()
    dev = torch.device("cuda", get_local_rank())
    torch.cuda.set_device(dev)
    pool = "mean" if a.pooling > 0 else "none"
    spec = EmbeddingTableConfig("t", ["f"], num_embeddings=a.rows, embedding_dim=a.dim, pooling=pool)
    emb = Embeddings([spec], device="meta" if world > 1 else dev,
                     optimizer=SparseOptimizer(kind=a.optimizer, lr=0.01))
    if world > 1:
        plan = TablePlan("t", a.sharding, ranks=list(range(world)),
                         owner=0 if a.sharding == "table_wise" else None, reason="bench")
        shard_embeddings(emb, {"t": plan}, rank, world, dev, comm=a.comm)
    L = a.pooling if a.pooling > 0 else a.ids
    g = torch.Generator().manual_seed(17 + rank)
    ids = [zipf_ids(a.rows, (a.batch, L), a.zipf, g).to(dev) for _ in range(3)]

    def fwd(i):
        return emb.lookup_groups({"f": ids[i % 3]}, [["f"]], dtype=torch.bfloat16)[0]

    for i in range(a.warmup):
        out = fwd(i)
        out.backward(torch.ones_like(out))
    torch.cuda.synchronize()
    ex = emb.executor
    if ex is not None and hasattr(ex, "take_phase_ms"):
        ex.take_phase_ms()
        ex.phase_ms = {}                      # phases of the timed steps only
    if world > 1:
        dist.barrier()
    ef = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
    eb = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
    gout = None
    for i in range(a.steps):
        ef[i][0].record()
        out = fwd(i)
        ef[i][1].record()
        if gout is None:
            gout = torch.randn_like(out)
        eb[i][0].record()
        out.backward(gout)
        eb[i][1].record()
    torch.cuda.synchronize()
    fwd_ms = sum(s.elapsed_time(e) for s, e in ef) / a.steps
    bwd_ms = sum(s.elapsed_time(e) for s, e in eb) / a.steps
    if ex is not None and hasattr(ex, "check"):
        ex.check()
    phases = ex.take_phase_ms() if ex is not None and hasattr(ex, "take_phase_ms") else {}
    # remote traffic: rows owned by other ranks (forward reads) and deduplicated
    # gradient rows sent to other owners (backward writes)
    n = ids[0].numel()
    if a.sharding == "row_wise":
        chunk = -(-a.rows // world)
        owners = [torch.div(x.reshape(-1), chunk, rounding_mode="floor") for x in ids]
    else:
        owners = [torch.zeros_like(x.reshape(-1)) for x in ids]
    remote_fwd = sum(int((o != rank).sum()) for o in owners) / 3 * a.dim * 4
    uniq = [torch.unique(x.reshape(-1)) for x in ids]
    remote_bwd = sum(int((torch.div(u, chunk, rounding_mode="floor") != rank).sum()) if a.sharding == "row_wise"
                     else int(u.numel()) * (rank != 0) for u in uniq) / 3 * (a.dim * 4 + 8)
    stats = torch.tensor([fwd_ms, bwd_ms, remote_fwd, remote_bwd], dtype=torch.float64, device=dev)
    if world > 1:
        mx = stats.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        fwd_ms, bwd_ms, remote_fwd, remote_bwd = mx.tolist()
    roof_f = remote_fwd / (a.link_gbs * 1e9) * 1e3
    roof_b = remote_bwd / (a.link_gbs * 1e9) * 1e3
    res = {"world": world, "comm": a.comm, "sharding": a.sharding, "rows": a.rows, "dim": a.dim,
           "ids_per_sample": L, "pooled": a.pooling > 0, "batch_per_rank": a.batch, "lookups_per_rank": n,
           "fwd_ms": round(fwd_ms, 3), "bwd_ms": round(bwd_ms, 3),
           "remote_fwd_GB": round(remote_fwd / 1e9, 3), "remote_bwd_GB": round(remote_bwd / 1e9, 3),
           "fwd_roofline_ms": round(roof_f, 3), "bwd_roofline_ms": round(roof_b, 3),
           "fwd_frac_of_link_roofline": round(roof_f / fwd_ms, 3) if fwd_ms > 0 and world > 1 else None,
           "bwd_frac_of_link_roofline": round(roof_b / bwd_ms, 3) if bwd_ms > 0 and world > 1 else None}
    if phases:
        res["bwd_phase_ms_rank0"] = {k: round(v / a.steps, 3) for k, v in phases.items() if k != "start"}
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return res


if __name__ == "__main__":
    main()

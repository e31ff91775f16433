#!/usr/bin/env python3
"""Headline benchmark: OneTrans v6-shaped training throughput on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|eager|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1)

Per rank: batch 2048 (global 2048 x N, weak scaling), synthetic Zipf data of
the benchmark v6 shapes, random-init weights, bf16 compute, fp32 embedding
tables row-wise sharded over the ranks, Adam sparse optimizer fused into the
lookup backward, AdamW dense with clipping.

Two measurements:
* ``value`` -- K training steps on device-resident batches, timed with CUDA
  events on the compute stream between barriers + synchronize; the max of
  the per-rank step time over ranks gives samples/s for the whole job.
* ``e2e``   -- K steps through ``TrainEngine.step_host`` (the public API):
  each step copies its packed batch from pinned host memory and reads the
  loss back to the host; wall clock between barriers, max over ranks.
Inputs exceed L2 (tables 7.7 GB, activations tens of GB per step), so no L2
flush is inserted.  nvidia-smi clocks are sampled during the timed region.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import tempfile
import sys
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIG = os.path.join(ROOT, "configs", "bench_onetrans_v6_b200.yaml")
PER_GPU_BATCH = 2048
METRIC = "train samples/sec (box, device-timed, max over ranks) at 1/2/4/8 B200; exposed a2a ms/step"
MODEL_DESC = "OneTrans v6-shaped: 8L d256 8hx32 NS16 pools 512/128/256 E128 Zipf1.05"


def _emit(obj: dict) -> None:
    print(json.dumps(obj), flush=True)


def _reference_arm(args) -> None:
    """Run the unmodified reference (baseline/_ref) if it can run here."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    why = None
    if not os.path.isdir(os.path.join(ref, "primus_dlrm")):
        why = "reference not installed under baseline/_ref"
    else:
        sys.path.insert(0, ref)
        try:
            import primus_dlrm.models.onetrans  # noqa: F401
        except Exception as e:  # torchrec / fbgemm_gpu are not installable offline
            why = (f"reference model path cannot import ({type(e).__name__}: {e}); torchrec and "
                   f"fbgemm_gpu are absent from the offline wheelhouse")
    if why is None:
        why = "reference training entry point requires torchrec DMP, not available offline"
    if int(os.environ.get("RANK", "0")) == 0:
        _emit({"impl": "reference", "unavailable": why})


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: list[int]):
        self.gpus = gpus
        self.proc = None
        # samples go to PD_CLOCKS_DIR when set (to keep them), else to the temp directory
        out_dir = os.environ.get("PD_CLOCKS_DIR") or tempfile.gettempdir()
        self.path = os.path.join(out_dir, f"clocks_{os.getpid()}.csv")

    def start(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", ",".join(str(g) for g in self.gpus)], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        mhz, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            p = [x.strip() for x in line.split(",")]
            if len(p) < 9:
                continue
            try:
                mhz.append(float(p[1]))
                mx.append(float(p[2]))
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(mhz)}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="native", choices=["native", "eager", "reference"])
    ap.add_argument("--config", default=CONFIG)
    ap.add_argument("--per-gpu-batch", type=int, default=PER_GPU_BATCH)
    ap.add_argument("--comm", default=None, choices=[None, "peer", "nccl"])
    ap.add_argument("--dense-strategy", default=None, choices=[None, "ddp", "fsdp", "zero2", "dmp"])
    args = ap.parse_args()
    if args.impl == "reference":
        _reference_arm(args)
        return
    args.warmup = max(args.warmup, 3)

    from primus_dlrm_b200.config import Config
    from primus_dlrm_b200.data.batch import PackedBatch
    from primus_dlrm_b200.data.synthetic import generate_batch
    from primus_dlrm_b200.ops import _ext
    from primus_dlrm_b200.parallel.setup import init_distributed, get_rank, get_world_size, get_local_rank
    from primus_dlrm_b200.parallel.build import build_training

    if args.impl == "eager":
        os.environ["PD_KERNELS"] = "eager"
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    init_distributed(timeout_s=600)
    rank, local = get_rank(), get_local_rank()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    torch.manual_seed(1234 + rank)

    cfg = Config.load(args.config)
    cfg.train.batch_size = args.per_gpu_batch * world
    model_desc = MODEL_DESC
    seq_len = cfg.sequence_length_total() + cfg.model.transformer.n_ns_tokens
    if cfg.model.model_type == "dlrm":
        mc = cfg.model
        model_desc = (f"{os.path.splitext(os.path.basename(args.config))[0]}: DLRM {mc.dlrm_layout} "
                      f"{len(mc.embedding_tables)} tables E{mc.embedding_dim}, bottom {mc.bottom_mlp_dims}, "
                      f"{mc.interaction_type} x{mc.dcn_num_cross_layers} rank {mc.dcn_low_rank}, top {mc.top_mlp_dims}")
        seq_len = 1
    elif os.path.abspath(args.config) != os.path.abspath(CONFIG):
        ot = cfg.model.transformer
        model_desc = (f"{os.path.splitext(os.path.basename(args.config))[0]}: {ot.n_layers}L d{ot.d_model} "
                      f"{ot.n_heads}hx{ot.d_model // ot.n_heads} NS{ot.n_ns_tokens} L_S{cfg.sequence_length_total()} "
                      f"E{cfg.model.embedding_dim}")
    if args.impl == "eager":
        cfg.train.kernels = "eager"
    if args.comm:
        cfg.distributed.comm = args.comm
    if args.dense_strategy:
        cfg.distributed.dense_strategy = args.dense_strategy
    model, engine = build_training(cfg, device)

    n_batches = 3
    packed = [PackedBatch(generate_batch(cfg, args.per_gpu_batch, seed=cfg.data.synthetic.seed + 1000 * rank + i))
              for i in range(n_batches)]
    dev_batches = [p.to_device(device) for p in packed]
    torch.cuda.synchronize()

    for i in range(args.warmup):
        engine.step(dev_batches[i % n_batches])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    C = _ext.core()
    sampler = ClockSampler(list(range(world))) if rank == 0 else None
    if sampler:
        sampler.start()
    l0 = C.launch_count() if C is not None else 0
    gemm = _ext.gemm()
    g0 = gemm.launch_count() if (gemm is not None and hasattr(gemm, "launch_count")) else 0
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ex = getattr(getattr(model, "emb", None), "executor", None)
    if ex is not None and hasattr(ex, "time_comm"):
        ex.time_comm = True
        ex.take_comm_ms()
    if ex is not None and hasattr(ex, "take_phase_ms"):
        ex.take_phase_ms()
        ex.phase_ms = {}                          # phases of the timed steps only
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev0.record()
    for i in range(args.steps):
        loss, _ = engine.step(dev_batches[i % n_batches])
    ev1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    launches = (C.launch_count() - l0) if C is not None else 0
    # the two extensions may share one counter (the dynamic linker merges the
    # header's counter when both are loaded); add the second only if distinct
    if gemm is not None and hasattr(gemm, "launch_count") and g0 != l0:
        launches += gemm.launch_count() - g0
    ms = ev0.elapsed_time(ev1) / args.steps
    a2a_ms = engine.exposed_comm_ms() / args.steps
    phases = {}
    if ex is not None and hasattr(ex, "take_phase_ms") and getattr(ex, "time_phases", False):
        phases = {k: round(v / args.steps, 3) for k, v in ex.take_phase_ms().items() if k != "start"}
    if ex is not None and hasattr(ex, "time_comm"):
        ex.time_comm = False

    # end-to-end through the public API (pinned H2D + loss D2H every step)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    last = 0.0
    for i in range(args.steps):
        last = engine.step_host(packed[i % n_batches])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2e_ms = (time.perf_counter() - t0) * 1000 / args.steps
    clocks = sampler.stop() if sampler else None
    # device error words of the peer-memory collectives (bounded waits that ran out)
    for obj in (ex, engine.grad_sync):
        if obj is not None and hasattr(obj, "check"):
            obj.check()

    peak_gb = torch.cuda.max_memory_allocated(device) / 2 ** 30
    stats = torch.tensor([ms, e2e_ms, float(launches), a2a_ms, peak_gb], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    ms, e2e_ms, launches, a2a_ms, peak_gb = stats.tolist()
    dense = cfg.distributed.dense_strategy if world > 1 else "single"
    par = {"ddp": "dp", "dmp": "dp", "fsdp": "fsdp", "zero2": "zero2-dp"}.get(dense, "dp")
    gb = args.per_gpu_batch * world
    if rank == 0:
        flops = model.get_num_flops_per_sample() if hasattr(model, "get_num_flops_per_sample") else 0.0
        value = gb / (ms / 1000.0)
        _emit({
            "metric": METRIC, "value": round(value, 1), "unit": "samples/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded Zipf ids, random-init weights)",
            "impl": args.impl,
            "config": {"model": model_desc, "global_batch": gb, "seq_len": seq_len,
                       "parallelism": f"{par}{world}" + (" + row-wise sharded tables" if world > 1 else ""),
                       "l2": "no flush: inputs exceed L2 (GB-scale tables, >10 GB activations per step)",
                       "embedding_optimizer": cfg.train.embedding_optimizer},
            "e2e": {"value": round(gb / (e2e_ms / 1000.0), 1), "unit": "samples/s",
                    "h2d_bytes_per_step": packed[0].nbytes, "d2h_bytes_per_step": 4,
                    "ms_per_step": round(e2e_ms, 3), "last_loss": round(last, 5)},
            "gpu_launches": int(launches),
            "exposed_a2a_ms_per_step": round(a2a_ms, 3),
            "exposed_a2a_note": ("device time of the sparse lookup+exchange (forward peer gather, backward "
                                 "route/dedup/push/barrier/update) on the compute stream; 0 on 1 GPU"),
            "tflops_per_gpu": round(flops * args.per_gpu_batch / (ms / 1000.0) / 1e12, 1),
            "clocks": clocks,
            "peak_mem_gib_max_rank": round(peak_gb, 2),
            **({"exchange_bwd_phase_ms_rank0": phases} if phases else {}),
        })
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

#!/usr/bin/env python3
"""Distributed training entry point (torchrun compatible); same flags as the
reference's ``scripts/run_distributed.py:273-311``.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 scripts/run_distributed.py \\
        --config configs/bench_onetrans_v6_b200.yaml --dense-strategy dmp --pipeline --skip-eval

``--dense-strategy dmp`` shards embedding tables (peer-memory exchange);
``ddp`` / ``fsdp`` keep the dense strategy and shard tables only when
``distributed.embedding_sharding.enabled``.  Additional flags: ``--comm``
(peer | nccl), ``--kernels`` (native | eager), ``--resume`` (a checkpoint
path or ``latest``), ``--eval-num-candidates``.
"""
from __future__ import annotations

import argparse
import logging
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

from primus_dlrm_b200.config import Config  # noqa: E402
from primus_dlrm_b200.parallel.setup import (  # noqa: E402
    barrier, cleanup, get_local_rank, get_rank, get_world_size, init_distributed, is_main_process,
)

_rank = os.environ.get("RANK", "?")
logging.basicConfig(level=logging.INFO, stream=sys.stdout, force=True,
                    format=f"%(asctime)s %(levelname)s [rank {_rank}][pid %(process)d] %(message)s")
logger = logging.getLogger("run_distributed")


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="Distributed OneTrans / DLRM training (B200)")
    p.add_argument("--config", required=True)
    p.add_argument("--data-root", default=None)
    p.add_argument("--dense-strategy", default="ddp", choices=["ddp", "fsdp", "zero2", "dmp"])
    p.add_argument("--embedding-sharding", default="auto",
                   choices=["auto", "table_wise", "row_wise", "data_parallel", "column_wise"])
    p.add_argument("--max-steps", type=int, default=0)
    p.add_argument("--run-name", default="dist_run")
    p.add_argument("--results-dir", default="results")
    p.add_argument("--log-interval", type=int, default=1000)
    p.add_argument("--skip-eval", action="store_true")
    p.add_argument("--trace", action="store_true")
    p.add_argument("--trace-steps", type=str, default="")
    p.add_argument("--trace-warmup", type=int, default=5)
    p.add_argument("--trace-active", type=int, default=10)
    p.add_argument("--trace-ranks", type=str, default="0")
    p.add_argument("--pipeline", action="store_true", help="overlap the next batch's H2D copy (dmp only)")
    p.add_argument("--attention-impl", default=None, choices=["sdpa", "fav2", "fav4", "turbo", "native"])
    # additive
    p.add_argument("--comm", default=None, choices=["peer", "nccl"])
    p.add_argument("--kernels", default=None, choices=["native", "eager"])
    p.add_argument("--resume", default=None, help="checkpoint path, or 'latest' in <results>/<run>/checkpoints")
    p.add_argument("--eval-num-candidates", type=int, default=None)
    return p.parse_args(argv)


def build_loader(config: Config, world: int, rank: int, data_root=None):
    """Synthetic infinite pipe, or the Yambda train dataset behind a DataLoader."""
    per_gpu = config.train.batch_size // world
    syn = config.data.synthetic
    if syn.enabled:
        from primus_dlrm_b200.data.synthetic import SyntheticDataPipe
        return SyntheticDataPipe(config, per_gpu, num_prebatched=syn.num_prebatched, seed=syn.seed + rank)
    from torch.utils.data import DataLoader, DistributedSampler

    from primus_dlrm_b200.data.dataset import DataPaths, LargeDatasetSampler, YambdaTrainDataset, collate_to_dict
    paths = DataPaths.from_config(config.data, data_root)
    ds = YambdaTrainDataset(config, paths)
    if len(ds) > 100_000_000:
        sampler = LargeDatasetSampler(ds, world, rank, shuffle=config.train.shuffle, seed=config.train.seed)
    else:
        sampler = DistributedSampler(ds, num_replicas=world, rank=rank, shuffle=config.train.shuffle)
    nw = config.data.num_workers
    return DataLoader(ds, batch_size=per_gpu, sampler=sampler, num_workers=nw, collate_fn=collate_to_dict,
                      pin_memory=True, drop_last=True, prefetch_factor=config.data.prefetch_factor if nw else None,
                      persistent_workers=nw > 0)


def build_eval_fn(config: Config, args, data_root=None):
    from primus_dlrm_b200.evaluation.metrics import evaluate_ranking, evaluate_ranking_peruser
    task = config.task_names[0]
    n_cand = args.eval_num_candidates or config.train.eval_num_candidates
    if config.data.synthetic.enabled:
        from primus_dlrm_b200.data.dataset import SyntheticEvalDataset
        ds = SyntheticEvalDataset(config, num_users=64, num_items_with_history=2000)

        def _eval(model, dev):
            rng = torch.Generator().manual_seed(0)
            cand = torch.randperm(ds.num_items, generator=rng)[:n_cand].numpy()
            return {"global-%d" % n_cand: evaluate_ranking(model, ds, dev, candidate_item_ids=cand,
                                                           ks=[10, 50, 100], task=task)}
        return _eval
    from primus_dlrm_b200.data.dataset import DataPaths, YambdaEvalDataset
    import numpy as np
    ds = YambdaEvalDataset(config, DataPaths.from_config(config.data, data_root))
    cand = np.argsort(-ds.item_popularity)[:n_cand]

    def _eval(model, dev):
        return {f"global-{n_cand}": evaluate_ranking(model, ds, dev, candidate_item_ids=cand, ks=[10, 50, 100],
                                                     task=task),
                "peruser-100": evaluate_ranking_peruser(model, ds, dev, ks=[10, 50, 100], task=task, top_n=100)}
    return _eval


def main(argv=None) -> None:
    args = parse_args(argv)
    init_distributed()
    rank, world, local = get_rank(), get_world_size(), get_local_rank()
    device = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")

    from primus_dlrm_b200.parallel.build import build_model
    from primus_dlrm_b200.parallel.wrapper import wrap_model
    from primus_dlrm_b200.training.checkpoint import latest_checkpoint, load_checkpoint
    from primus_dlrm_b200.training.engine import TrainEngine
    from primus_dlrm_b200.training.runtime import apply_cli_overrides, configure_runtime, log_resolved_config
    from primus_dlrm_b200.training.tracer import parse_trace_ranks
    from primus_dlrm_b200.training.trainer import DistributedTrainer

    config = Config.load(args.config)
    apply_cli_overrides(config, args)
    if args.dense_strategy == "dmp":
        config.distributed.embedding_sharding.enabled = True
    configure_runtime(config.train)
    if is_main_process():
        log_resolved_config(config, args.config)
    torch.manual_seed(config.train.seed + rank)
    run_dir = Path(args.results_dir) / args.run_name
    if is_main_process():
        (run_dir / "logs").mkdir(parents=True, exist_ok=True)
        fh = logging.FileHandler(run_dir / "logs" / "train.log")
        fh.setFormatter(logging.Formatter("%(asctime)s %(levelname)s %(message)s"))
        logging.getLogger().addHandler(fh)

    loader = build_loader(config, world, rank, args.data_root)
    torch.manual_seed(config.train.seed)   # identical dense init on every rank
    model = build_model(config, device=device, meta_device=world > 1)
    model, grad_sync = wrap_model(model, device, config)
    total = config.train.epochs * (len(loader) if hasattr(loader, "__len__") else 10_000_000)
    engine = TrainEngine(model, config, device, grad_sync=grad_sync, total_steps=total)
    if args.resume:
        ck = latest_checkpoint(run_dir) if args.resume == "latest" else Path(args.resume)
        if ck is not None:
            ckpt = load_checkpoint(ck, model, engine)
            logger.info("resumed from %s (epoch %s, step %s)", ck, ckpt.get("epoch"), ckpt.get("global_step"))
    eval_fn = None if args.skip_eval else build_eval_fn(config, args, args.data_root)
    barrier()
    config.train.checkpoint_dir = str(run_dir)
    trainer = DistributedTrainer(
        model, engine, loader, config, device, eval_fn=eval_fn, max_steps=args.max_steps,
        log_interval=args.log_interval, trace=args.trace,
        trace_steps=[int(s) for s in args.trace_steps.split(",") if s.strip()] or None,
        trace_warmup=args.trace_warmup, trace_active=args.trace_active,
        trace_ranks=parse_trace_ranks(args.trace_ranks), run_dir=run_dir, pipeline=args.pipeline)
    trainer.train()
    ex = getattr(getattr(model, "emb", None), "executor", None)
    if ex is not None and hasattr(ex, "check"):
        ex.check()
    cleanup()
    if is_main_process():
        logger.info("Training complete.")


if __name__ == "__main__":
    main()

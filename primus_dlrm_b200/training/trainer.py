"""Training loop (``primus_dlrm/training/dist_trainer.py:243-756`` and the
single-GPU ``primus_dlrm/training/trainer.py``).

``DistributedTrainer`` drives ``TrainEngine`` over epochs with:

* ``pipeline=True`` -- the next batch's host->device copy runs on a copy
  stream (one packed pinned buffer per batch) while the current step
  computes.  (The reference's 3-stage TorchRec pipeline also overlaps the
  input-id all-to-all; the peer-memory lookup has no input all-to-all.)
* log lines every ``log_interval`` steps with the reference's fields: loss,
  lr, global / window throughput, per-task losses, TFLOPS/GPU and MFU from
  the analytic FLOP count, memory, plus the device time of the sparse
  exchange;
* a torch.profiler window tracer on selected ranks;
* epoch-end checkpoint (rank-0 assembled, atomic) and evaluation;
* a host watchdog that ends the process when a step does not finish within
  ``train.step_timeout_s`` (0 = off), so a dead peer surfaces as an error;
* peer heartbeats (``parallel.health``): a rank that raised or went silent
  stops the others between steps with ``PeerFailure``;
* an optional NaN/Inf guard that skips the optimizer step.
"""
from __future__ import annotations

import logging
import os
import threading
import time
from pathlib import Path

import torch
import torch.distributed as dist

from primus_dlrm_b200.config import Config
from primus_dlrm_b200.data.batch import DeviceBatchStager, PackedBatch
from primus_dlrm_b200.parallel.health import HealthMonitor
from primus_dlrm_b200.parallel.setup import barrier, get_rank, get_world_size, is_main_process
from primus_dlrm_b200.training.checkpoint import save_checkpoint
from primus_dlrm_b200.training.engine import TrainEngine
from primus_dlrm_b200.training.tracer import Tracer
from primus_dlrm_b200.utils.model_params import log_param_summary

logger = logging.getLogger(__name__)

PEAK_FLOPS = {"B200": {"bf16": 2250e12, "tf32": 1100e12, "fp32": 75e12},
              "H100": {"bf16": 990e12, "tf32": 495e12, "fp32": 67e12},
              "A100": {"bf16": 312e12, "tf32": 156e12, "fp32": 19.5e12}}


def gpu_peak_flops(dtype: str = "bf16") -> float:
    if not torch.cuda.is_available():
        return 0.0
    name = torch.cuda.get_device_name(0)
    for k, v in PEAK_FLOPS.items():
        if k in name:
            return v.get(dtype, v["bf16"])
    return PEAK_FLOPS["B200"][dtype]


def system_metrics(device) -> str:
    parts = []
    if torch.cuda.is_available() and torch.device(device).type == "cuda":
        free, total = torch.cuda.mem_get_info(device)
        parts.append(f"gpu_mem_used={(total - free) / 2**30:.1f}GB/{total / 2**30:.0f}GB")
        parts.append(f"torch_max_alloc={torch.cuda.max_memory_allocated(device) / 2**30:.1f}GB")
    try:
        import psutil
        parts.append(f"rss={psutil.Process().memory_info().rss / 2**30:.1f}GB")
    except ImportError:
        pass
    return " ".join(parts)


def gather_max_gpu_memory(device) -> str:
    """Max GPU memory in use over all ranks (a collective: every rank calls it)."""
    if not (torch.cuda.is_available() and dist.is_initialized()):
        return ""
    free, total = torch.cuda.mem_get_info(device)
    t = torch.tensor([float(total - free)], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return f"max_gpu_mem_all_ranks={t.item() / 2**30:.1f}GB"


class Watchdog:
    """Host thread: once armed by the first ``kick()`` (the first step may
    include one-time setup), if ``kick()`` is not called again within
    ``timeout_s`` seconds ``on_timeout`` runs (default: log and exit the
    process with code 17)."""

    def __init__(self, timeout_s: float, on_timeout=None):
        self.timeout_s = timeout_s
        self.on_timeout = on_timeout or self._default
        self._last = None
        self._stop = threading.Event()
        self.fired = False
        self._t = threading.Thread(target=self._run, daemon=True)
        if timeout_s > 0:
            self._t.start()

    def _default(self) -> None:
        logger.error("watchdog: no training step finished in %.1f s on rank %d; exiting", self.timeout_s,
                     get_rank())
        os._exit(17)

    def kick(self) -> None:
        self._last = time.monotonic()

    def _run(self) -> None:
        while not self._stop.wait(min(1.0, self.timeout_s / 4)):
            last = self._last
            if last is not None and time.monotonic() - last > self.timeout_s:
                self.fired = True
                self.on_timeout()
                return

    def stop(self) -> None:
        self._stop.set()


class DistributedTrainer:
    def __init__(self, model, engine: TrainEngine, train_loader, config: Config, device: torch.device,
                 eval_fn=None, max_steps: int = 0, log_interval: int = 1000, trace: bool = False,
                 trace_steps: list[int] | None = None, trace_warmup: int = 5, trace_active: int = 10,
                 trace_ranks: set[int] | None = None, run_dir: str | Path | None = None, pipeline: bool = False):
        self.model = model
        self.engine = engine
        self.loader = train_loader
        self.config = config
        self.device = torch.device(device)
        self.eval_fn = eval_fn
        self.max_steps = max_steps
        self.log_interval = max(int(log_interval), 1)
        self.pipeline = pipeline and self.device.type == "cuda"
        self.run_dir = Path(run_dir or config.train.checkpoint_dir)
        self.ckpt_dir = self.run_dir / "checkpoints"
        inner = getattr(model, "module", model)
        self.flops_per_sample = inner.get_num_flops_per_sample() if hasattr(inner, "get_num_flops_per_sample") else 0.0
        self.tracer = None
        on_rank = trace_ranks is None or get_rank() in trace_ranks
        if trace and on_rank:
            self.tracer = Tracer(self.run_dir / "trace", trace_steps=trace_steps, warmup=trace_warmup,
                                 active=trace_active, rank=get_rank())
        self.watchdog = Watchdog(config.train.step_timeout_s)
        self.health = HealthMonitor(config.train.heartbeat_timeout_s)
        if is_main_process():
            log_param_summary(model, config, get_world_size())
            if self.flops_per_sample:
                logger.info("Estimated %.1f GFLOP/sample (fwd+bwd), peak %.0f TFLOPS", self.flops_per_sample / 1e9,
                            gpu_peak_flops("bf16" if config.train.bf16 else "fp32") / 1e12)

    # ------------------------------------------------------------------
    def _device_batches(self):
        """Yield device batches; with pipelining the next copy overlaps compute."""
        it = iter(self.loader)
        if not self.pipeline:
            for b in it:
                if isinstance(b, PackedBatch):
                    yield b.to_device(self.device)
                else:
                    yield {k: (v.to(self.device, non_blocking=True) if isinstance(v, torch.Tensor) else v)
                           for k, v in b.items()}
            return
        stager = None
        try:
            nxt = next(it)
        except StopIteration:
            return
        while True:
            packed = nxt if isinstance(nxt, PackedBatch) else PackedBatch(nxt)
            if stager is None or stager.bufs[0].numel() < packed.nbytes:
                stager = DeviceBatchStager(self.device, packed.nbytes)
            stager.stage(packed)
            try:
                nxt = next(it)
            except StopIteration:
                yield stager.get()
                return
            yield stager.get()

    def train(self) -> dict:
        try:
            return self._train()
        except BaseException as e:
            self.health.report_failure(f"{type(e).__name__}: {e}")
            self.watchdog.stop()
            raise
        finally:
            self.health.stop()

    def _train(self) -> dict:
        tc = self.config.train
        world = get_world_size()
        per_gpu = tc.batch_size // max(world, 1)
        logger.info("Training: %s, global batch %d (%d per rank), world %d",
                    "pipelined" if self.pipeline else "sequential", tc.batch_size, per_gpu, world)
        peak = gpu_peak_flops("bf16" if tc.bf16 else ("tf32" if tc.allow_tf32 else "fp32"))
        last_loss = torch.zeros((), device=self.device)
        history = []
        for epoch in range(tc.epochs):
            sampler = getattr(self.loader, "sampler", None)
            if hasattr(sampler, "set_epoch"):
                sampler.set_epoch(epoch)
            t0 = tw = time.time()
            n = 0
            epoch_loss = torch.zeros((), device=self.device)
            for batch in self._device_batches():
                self.health.check()          # a failed peer stops us before this step's launches
                loss, task_losses = self.engine.step(batch)
                self.health.beat(self.engine.global_step)
                self.watchdog.kick()
                if self.tracer:
                    self.tracer.step()
                epoch_loss += loss
                last_loss = loss
                n += 1
                step = self.engine.global_step - 1
                if step % self.log_interval == 0:
                    mem = gather_max_gpu_memory(self.device) if tc.log_max_gpu_memory else ""
                    comm_ms = self.engine.exposed_comm_ms()
                    lv = float(loss)
                    history.append(lv)
                    if is_main_process():
                        now = time.time()
                        thr = n * per_gpu * world / max(now - t0, 1e-9)
                        wthr = min(self.log_interval, n) * per_gpu * world / max(now - tw, 1e-9)
                        tfl = self.flops_per_sample * wthr / world / 1e12 if self.flops_per_sample else 0.0
                        mfu = 100 * tfl * 1e12 / peak if peak else 0.0
                        lr = self.engine.optimizer.param_groups[0]["lr"]
                        tl = " | ".join(f"{k}={float(v.detach()):.4f}" for k, v in task_losses.items())
                        logger.info(f"epoch={epoch} step={step} | loss={lv:.4f} | lr={lr:.6f} | "
                                    f"global_throughput={thr:.0f} samples/s | window_throughput={wthr:.0f} "
                                    f"samples/s (over {self.log_interval} steps) | {tl} | tflops/gpu={tfl:.1f} "
                                    f"mfu={mfu:.1f}% | sparse_exchange_ms={comm_ms:.2f} | "
                                    f"{system_metrics(self.device)}" + (f" | {mem}" if mem else ""))
                        tw = now
                if self.max_steps and self.engine.global_step >= self.max_steps:
                    break
            dt = time.time() - t0
            if is_main_process():
                logger.info(f"=== Epoch {epoch} done === avg_loss={float(epoch_loss) / max(n, 1):.4f} | "
                            f"last_loss={float(last_loss):.4f} | time={dt:.1f}s | "
                            f"global_throughput={n * per_gpu * world / max(dt, 1e-9):.0f} samples/s")
            barrier()
            if tc.save_checkpoint:
                save_checkpoint(self.ckpt_dir / f"epoch_{epoch}.pt", self.model, epoch, self.engine.global_step,
                                engine=self.engine, config=self.config)
            elif is_main_process():
                logger.info("Checkpoint saving is disabled (save_checkpoint=False)")
            if self.eval_fn is not None and (epoch + 1) % max(tc.eval_interval, 1) == 0:
                self.run_eval()
            barrier()
            if self.max_steps and self.engine.global_step >= self.max_steps:
                break
        if self.tracer:
            self.tracer.stop()
            logger.info("[rank %d] traces in %s (%d files)", get_rank(), self.tracer.trace_dir,
                        len(self.tracer.trace_files))
        self.watchdog.stop()
        return {"loss_history": history, "global_step": self.engine.global_step}

    def run_eval(self) -> dict | None:
        """Every rank runs the eval function (a sharded model's lookups are
        collective); rank 0 logs the metrics."""
        self.model.eval()
        with torch.no_grad():
            metrics = self.eval_fn(self.model, self.device)
        self.model.train()
        if is_main_process() and metrics:
            for name, m in metrics.items():
                logger.info(f"  [{name}] " + " | ".join(
                    f"{k}={v:.4f}" if isinstance(v, float) else f"{k}={v}" for k, v in sorted(m.items())))
        return metrics

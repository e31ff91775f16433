"""Distributed wrapping of a model (``primus_dlrm/distributed/wrapper.py:27-79``).

``wrap_model(model, device, config) -> (model, grad_sync)``:

* embedding tables are sharded by the plan (``parallel.planner``) whenever
  ``distributed.embedding_sharding.enabled`` or ``dense_strategy == "dmp"``;
  otherwise they are replicated (data-parallel with a sparse gradient
  all-gather), which is what the reference's plain DDP run does;
* dense parameters are broadcast from rank 0 and their gradients are
  synchronised over NVLink peer memory on CUDA (``distributed.comm: peer``):
  ``PeerGradSync`` (``ddp`` / ``dmp``: two-shot all-reduce of the flat
  gradient arena by slice kernels) or ``PeerShardedGradSync`` (``zero2``:
  slice reduce-scatter, AdamW on this rank's 1/W slice, parameter
  all-gather -- optimizer state and gradients sharded, parameters
  replicated). With ``comm: nccl`` (and on CPU / gloo) the same strategies
  run as NCCL collectives (``FlatGradSync`` / ``ShardedGradSync``), the
  baseline;
* ``fsdp`` shards the parameters themselves (``parallel.fsdp``: per-block
  units, all-gather one block ahead, fp32 master / gradient / moment shards).

``distributed.comm`` picks the sparse exchange: ``peer`` (NVLink peer-memory
kernels, CUDA) or ``nccl`` (collective baseline; also the CPU/gloo path).
"""
from __future__ import annotations

import logging
import os

import torch
import torch.distributed as dist
import torch.nn as nn

from primus_dlrm_b200.parallel.planner import build_topology, log_plan, plan_tables
from primus_dlrm_b200.parallel.setup import get_rank, get_world_size
from primus_dlrm_b200.parallel.sharded_embedding import shard_embeddings

logger = logging.getLogger(__name__)


class FlatGradSync:
    """Average the flat dense-gradient arena over ranks (bucketed all-reduce)."""

    def __init__(self, group=None, bucket_mb: float = 256.0):
        self.group = group
        self.world = dist.get_world_size(group)
        self.bucket = int(bucket_mb * 2 ** 20 / 4)

    def sync(self, flat_grad: torch.Tensor) -> None:
        n = flat_grad.numel()
        works = []
        for s in range(0, n, self.bucket):
            works.append(dist.all_reduce(flat_grad[s:s + self.bucket], group=self.group, async_op=True))
        for w in works:
            w.wait()
        flat_grad.mul_(1.0 / self.world)


class ShardedGradSync:
    """ZeRO-2: reduce-scatter gradients so each rank owns 1/W of them,
    update that slice, all-gather the parameters (``zero2`` strategy)."""

    sharded = True

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def shard_range(self, n: int) -> tuple[int, int]:
        per = -(-n // self.world)
        per = (per + 63) // 64 * 64
        a = min(self.rank * per, n)
        return a, min(a + per, n)

    def sync(self, flat_grad: torch.Tensor) -> None:
        n = flat_grad.numel()
        per = (-(-n // self.world) + 63) // 64 * 64
        pad = per * self.world - n
        g = torch.nn.functional.pad(flat_grad, (0, pad)) if pad else flat_grad
        out = torch.empty(per, dtype=g.dtype, device=g.device)
        dist.reduce_scatter_tensor(out, g, group=self.group)
        a, b = self.shard_range(n)
        flat_grad.zero_()
        flat_grad[a:b].copy_(out[: b - a]).mul_(1.0 / self.world)

    def gather_params(self, flat_data: torch.Tensor) -> None:
        n = flat_data.numel()
        per = (-(-n // self.world) + 63) // 64 * 64
        a, b = self.shard_range(n)
        mine = torch.zeros(per, dtype=flat_data.dtype, device=flat_data.device)
        mine[: b - a] = flat_data[a:b]
        full = torch.empty(per * self.world, dtype=flat_data.dtype, device=flat_data.device)
        dist.all_gather_into_tensor(full, mine, group=self.group)
        flat_data.copy_(full[:n])


class _PeerDense:
    """Shared machinery of the peer-memory dense collectives: a flat fp32
    buffer mapped into every rank, a signal pad for bounded barriers, and the
    64-element aligned slice boundaries (rank r owns [bounds[r], bounds[r+1]))."""

    def __init__(self, numel: int, device: torch.device, group=None, timeout_s: float = 60.0):
        from primus_dlrm_b200.ops import _ext
        from primus_dlrm_b200.parallel.sharded_embedding import SymmetricBuffer
        self.C = _ext.core()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.numel = int(numel)
        per = (-(-self.numel // self.world) + 63) // 64 * 64
        self.per = per
        b = [min(r * per, self.numel) for r in range(self.world + 1)]
        self.bounds = torch.tensor(b, dtype=torch.int64, device=device)
        self.slice = (b[self.rank], b[self.rank + 1])
        self.mem = SymmetricBuffer(per * self.world * 4, device, self.rank, self.world, group)
        self.buf = self.mem.local[: self.numel * 4].view(torch.float32)
        self.ptrs = torch.tensor(self.mem.ptrs, dtype=torch.int64)
        self.pads = SymmetricBuffer(64 * 8, device, self.rank, self.world, group)
        self.pad_ptrs = torch.tensor(self.pads.ptrs, dtype=torch.int64)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.timeout_ns = int(timeout_s * 1e9)
        self.epoch = 0

    def barrier(self) -> None:
        self.epoch += 1
        self.C.signal_barrier(self.pad_ptrs, self.rank, self.epoch, self.timeout_ns, self.err)

    def check(self) -> None:
        code = int(self.err.item())
        if code:
            raise RuntimeError(f"peer dense collective on rank {self.rank}: error word {code} "
                               f"(2 = a peer did not reach a barrier in time)")

    def reduce_scatter(self, scale: float) -> None:
        a, b = self.slice
        self.barrier()
        self.C.peer_reduce_slice(self.ptrs, self.rank, self.buf, a, b, scale, 0)

    def all_gather(self) -> None:
        self.barrier()
        self.C.peer_gather_slices(self.ptrs, self.rank, self.buf, self.bounds, 0, 0)
        self.barrier()


class PeerGradSync(_PeerDense):
    """DDP gradient averaging over NVLink peer memory (two-shot all-reduce:
    each rank reduces its 1/W slice from every peer's arena, then gathers the
    other slices). The flat gradient arena itself lives in the shared buffer
    (``bind``), so backward writes straight into memory the peers read.

    Overlap with the backward (the reference's bucketed DDP,
    ``primus_dlrm/distributed/wrapper.py:61-64``): the arena is cut into
    buckets of about ``PD_DDP_BUCKET_MB`` (default 32) MB in reverse parameter
    order, the order in which the backward produces the gradients. A
    post-accumulate-grad hook on every parameter counts the gradients a bucket
    still waits for; when the count reaches zero the bucket's reduce-scatter
    and all-gather are launched on a side stream, right behind the kernels
    that wrote its last gradient. Buckets launch strictly in index order, so
    every rank issues the same sequence of collectives. ``finish`` launches
    the buckets whose parameters got no gradient this step and makes the
    compute stream wait for the side stream.
    """

    BLOCKS = 32          # CTAs per overlapped reduce / gather: the backward keeps the rest of the GPU

    def __init__(self, numel: int, device: torch.device, group=None, timeout_s: float = 60.0,
                 bucket_mb: float | None = None):
        super().__init__(numel, device, group, timeout_s)
        self._side = None
        self.bucket_mb = float(os.environ.get("PD_DDP_BUCKET_MB", "32")) if bucket_mb is None else bucket_mb
        self.buckets: list[tuple[int, int, int, int, torch.Tensor]] = []   # (lo, hi, a, b, bounds)
        self._bucket_params: list[int] = []
        self._hooks = []
        self._armed = False
        self._left: list[int] = []
        self._launched = 0

    def bind(self, flat) -> None:
        self.buf.copy_(flat.grad)
        flat.grad = self.buf
        flat.zero_grad()
        if hasattr(flat, "params") and hasattr(flat, "offsets"):
            self._build_buckets(flat)

    def _build_buckets(self, flat) -> None:
        cap = max(int(self.bucket_mb * 2 ** 20 / 4), 64)
        sizes = [(p.numel() + 63) // 64 * 64 for p in flat.params]
        groups, cur, size = [], [], 0
        for i in reversed(range(len(flat.params))):
            cur.append(i)
            size += sizes[i]
            if size >= cap:
                groups.append(cur)
                cur, size = [], 0
        if cur:
            groups.append(cur)
        dev = self.buf.device
        for k, idx in enumerate(groups):
            lo = min(flat.offsets[i] for i in idx)
            hi = min(max(flat.offsets[i] + sizes[i] for i in idx), self.numel)
            per = (-(-(hi - lo) // self.world) + 63) // 64 * 64
            b = [min(lo + r * per, hi) for r in range(self.world + 1)]
            self.buckets.append((lo, hi, b[self.rank], b[self.rank + 1],
                                 torch.tensor(b, dtype=torch.int64, device=dev)))
            self._bucket_params.append(len(idx))
            for i in idx:
                self._hooks.append(flat.params[i].register_post_accumulate_grad_hook(
                    lambda _p, k=k: self._on_grad(k)))

    def sync(self, flat_grad: torch.Tensor) -> None:
        if flat_grad.data_ptr() != self.buf.data_ptr():
            self.buf.copy_(flat_grad)
        self.reduce_scatter(1.0 / self.world)
        self.all_gather()
        if flat_grad.data_ptr() != self.buf.data_ptr():
            flat_grad.copy_(self.buf)

    # -- overlap with the backward -----------------------------------------
    def begin(self) -> bool:
        """Arm the bucket hooks for one backward; False when there are no buckets."""
        if not self.buckets or not self.buf.is_cuda:
            return False
        if self._side is None:
            self._side = torch.cuda.Stream(self.buf.device)
        self._left = list(self._bucket_params)
        self._launched = 0
        self._armed = True
        return True

    def _on_grad(self, k: int) -> None:
        if not self._armed:
            return
        self._left[k] -= 1
        while self._launched < len(self.buckets) and self._left[self._launched] <= 0:
            self._launch(self._launched)
            self._launched += 1

    def _launch(self, k: int) -> None:
        lo, hi, a, b, bounds = self.buckets[k]
        self._side.wait_stream(torch.cuda.current_stream(self.buf.device))
        with torch.cuda.stream(self._side):
            self.barrier()                                  # every rank's bucket k is final
            self.C.peer_reduce_slice(self.ptrs, self.rank, self.buf, a, b, 1.0 / self.world, self.BLOCKS)
            self.barrier()                                  # every slice of bucket k is reduced
            self.C.peer_gather_slices(self.ptrs, self.rank, self.buf, bounds, hi - lo, self.BLOCKS)

    def finish(self) -> bool:
        """Launch the buckets not started during the backward, then make the
        compute stream wait for all of them. False if ``begin`` was not called."""
        if not self._armed:
            return False
        self._armed = False
        for k in range(self._launched, len(self.buckets)):
            self._launch(k)
        self._launched = len(self.buckets)
        with torch.cuda.stream(self._side):
            self.barrier()               # peers have finished reading this rank's arena
        torch.cuda.current_stream(self.buf.device).wait_stream(self._side)
        return True


class PeerShardedGradSync(_PeerDense):
    """ZeRO-2 sharding over peer memory (``zero2``): gradients are
    reduce-scattered by the slice kernel (each rank keeps the average of its
    slice), AdamW updates that slice, and parameters are all-gathered from
    the owners' arenas. Parameters and gradients both live in shared buffers."""

    sharded = True

    def __init__(self, numel: int, device: torch.device, group=None, timeout_s: float = 60.0):
        super().__init__(numel, device, group, timeout_s)
        self.params = _PeerDense(numel, device, group, timeout_s)

    def shard_range(self, n: int) -> tuple[int, int]:
        return self.slice

    def bind(self, flat) -> None:
        self.buf.copy_(flat.grad)
        flat.grad = self.buf
        self.params.buf.copy_(flat.data)
        flat.data = self.params.buf
        flat.rebind_all()
        flat.zero_grad()

    def sync(self, flat_grad: torch.Tensor) -> None:
        if flat_grad.data_ptr() != self.buf.data_ptr():
            self.buf.copy_(flat_grad)
        self.reduce_scatter(1.0 / self.world)
        # peers read this arena during the reduction; wait before it is reused
        self.barrier()

    def gather_params(self, flat_data: torch.Tensor) -> None:
        if flat_data.data_ptr() != self.params.buf.data_ptr():
            self.params.buf.copy_(flat_data)
        self.params.all_gather()
        if flat_data.data_ptr() != self.params.buf.data_ptr():
            flat_data.copy_(self.params.buf)

    def check(self) -> None:
        super().check()
        self.params.check()


def all_gather_slices(flat: torch.Tensor, group=None) -> None:
    """Fill every rank's copy of ``flat`` from the owners of its 64-aligned
    1/W slices (the slice layout of ``ShardedGradSync`` and ``_PeerDense``);
    used for checkpoints of the ``zero2`` optimizer state."""
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    n = flat.numel()
    per = (-(-n // world) + 63) // 64 * 64
    a, b = min(rank * per, n), min(rank * per + per, n)
    mine = torch.zeros(per, dtype=flat.dtype, device=flat.device)
    mine[: b - a] = flat[a:b]
    full = torch.empty(per * world, dtype=flat.dtype, device=flat.device)
    dist.all_gather_into_tensor(full, mine, group=group)
    flat.copy_(full[:n])


def broadcast_dense(model: nn.Module, group=None) -> None:
    for p in model.parameters():
        if p.requires_grad:
            dist.broadcast(p.data, src=0, group=group)


def wrap_model(model: nn.Module, device: torch.device, config, group=None):
    world = get_world_size()
    rank = get_rank()
    dc = config.distributed
    if world <= 1:
        return model.to(device), None
    inner = getattr(model, "module", model)
    emb = getattr(inner, "emb", None)
    if emb is not None:
        comm = dc.comm if device.type == "cuda" else "nccl"
        if dc.embedding_sharding.enabled or dc.dense_strategy == "dmp":
            plans = plan_tables(config, world, build_topology(config, world))
        else:
            from primus_dlrm_b200.parallel.planner import TablePlan
            plans = {t.name: TablePlan(t.name, "data_parallel", ranks=list(range(world)), reason="ddp")
                     for t in emb.tables()}
        if rank == 0:
            log_plan(plans)
        shard_embeddings(emb, plans, rank, world, device, comm=comm, group=group,
                         seed=config.train.seed, init=config.model.embedding_init)
    model = model.to(device)
    broadcast_dense(model, group)
    peer = device.type == "cuda" and dc.comm == "peer"
    if dc.dense_strategy not in ("fsdp", "zero2", "ddp", "dmp"):
        raise ValueError(f"Unknown dense_strategy: {dc.dense_strategy!r}")
    if dc.dense_strategy == "fsdp":
        from primus_dlrm_b200.parallel.fsdp import shard_dense
        sync = shard_dense(model, device, group, torch.bfloat16 if config.train.bf16 else None)
    elif peer:
        # sized by the flat arena the engine builds (bind() is called with it)
        sync = _LazyPeerSync(device, group, sharded=dc.dense_strategy == "zero2")
    elif dc.dense_strategy == "zero2":
        sync = ShardedGradSync(group)
    else:
        sync = FlatGradSync(group)
    logger.info("wrapped for %d ranks: dense=%s embeddings=%s comm=%s", world, dc.dense_strategy,
                "sharded" if emb is not None and emb.sharded else "none", dc.comm)
    return model, sync


class _LazyPeerSync:
    """Placeholder until the engine's flat arena exists: ``bind(flat)``
    builds the peer collective of the right size and becomes it."""

    def __init__(self, device, group, sharded: bool):
        self.device, self.group, self._sharded = device, group, sharded
        self.impl = None

    @property
    def sharded(self) -> bool:
        return self._sharded

    def bind(self, flat) -> None:
        cls = PeerShardedGradSync if self._sharded else PeerGradSync
        self.impl = cls(flat.numel, self.device, self.group)
        self.impl.bind(flat)

    def __getattr__(self, name):
        impl = self.__dict__.get("impl")
        if impl is None:
            raise AttributeError(f"peer gradient sync used before bind(): {name}")
        return getattr(impl, name)


def _has_meta_dense(model: nn.Module) -> bool:
    return any(p.device.type == "meta" and p.requires_grad for p in model.parameters())


def is_dmp(model: nn.Module) -> bool:
    inner = getattr(model, "module", model)
    emb = getattr(inner, "emb", None)
    return bool(emb is not None and getattr(emb, "sharded", False))

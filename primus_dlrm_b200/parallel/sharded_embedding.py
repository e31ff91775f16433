"""Model-parallel embedding tables across ranks.

Replaces TorchRec DMP's sharded EC/EBC (``primus_dlrm/distributed/wrapper.py:110-257``)
and the reference's native fallback (``primus_dlrm/models/sharded_embedding.py``).

Placement (``parallel.planner``): row-wise (rows ``[r*chunk, (r+1)*chunk)`` on
rank r), table-wise (whole table on one rank), column-wise (rank c holds
columns ``[c*E/W, (c+1)*E/W)``; lookups read one column block from every
rank) and data-parallel (replicated).

Two exchange backends share the same placement and semantics:

* ``peer`` (product, CUDA only) -- every table shard is allocated in
  IPC-exportable device memory and mapped into every rank.  Forward: the
  ordinary gather kernel reads each row straight from the owner's HBM over
  NVLink (peer loads; no id or row all-to-all, no host sync).  Backward:
  keys are routed by owner, gradients are reduced per unique row locally
  (Zipf dedup), pushed into the owner's receive slab with peer stores,
  a signal-pad barrier publishes them, and the owner applies the fused
  sparse optimizer.  A second barrier orders those updates before any rank's
  next lookup.
* ``a2a`` (baseline; CPU/gloo and NCCL) -- the reference program shape:
  ``all_to_all_single`` of ids to owners, owner-side lookup, rows back; the
  backward sends per-id gradients to owners.  Replicated tables all-gather
  their (row, grad) lists.
"""
from __future__ import annotations

import os

import logging
import math
import time

import torch
import torch.distributed as dist

from primus_dlrm_b200.ops import _ext
from primus_dlrm_b200.ops.embedding import (
    LookupSpec, TableShard, _by_dim, _eager_pooled, _eager_rows, _launch_tables, _native_forward,
    _slot_view, _table_meta, eager_sparse_update,
)
from primus_dlrm_b200.parallel.planner import TablePlan

logger = logging.getLogger(__name__)

_OWNER_SHIFT = 44
_KEY_MASK = (1 << _OWNER_SHIFT) - 1
_KIND_CODE = {"row_wise": 0, "table_wise": 1, "column_wise": 1, "data_parallel": 2}


# ---------------------------------------------------------------------------
# placement
# ---------------------------------------------------------------------------

def _init_local(w: torch.Tensor, rows: int, seed: int, how: str) -> None:
    g = torch.Generator(device=w.device).manual_seed(seed)
    if how == "normal":
        w.normal_(0.0, 1.0, generator=g)
    else:
        b = math.sqrt(1.0 / max(rows, 1))
        w.uniform_(-b, b, generator=g)


def _alloc_weight(rows: int, dim: int, device: torch.device, shared: bool) -> torch.Tensor:
    if shared and rows > 0:
        buf = _ext.core().alloc_shared(rows * dim * 4, device.index)
        return buf.view(torch.float32).view(rows, dim)
    return torch.zeros(rows, dim, dtype=torch.float32, device=device)


def shard_embeddings(emb, plans: dict[str, TablePlan], rank: int, world: int, device: torch.device,
                     comm: str = "peer", group=None, seed: int = 1234, init: str = "uniform") -> None:
    """Materialise this rank's shards of every table of ``emb`` (built on the
    meta device) and install the exchange executor."""
    device = torch.device(device)
    shared = comm == "peer"
    for ti, t in enumerate(emb.tables()):
        p = plans[t.name]
        rows, dim = t.num_embeddings, t.embedding_dim
        t.plan = p
        if p.kind == "row_wise":
            chunk = -(-rows // world)
            r0 = min(rank * chunk, rows)
            lr = max(min(chunk, rows - r0), 0)
            w = _alloc_weight(lr, dim, device, shared)
            _init_local(w, rows, seed * 1000 + ti * 64 + rank, init)
            t.weight = torch.nn.Parameter(w, requires_grad=False)
            t.shard = TableShard(name=t.name, rows=rows, dim=dim, weight=w, local_row0=r0, chunk=chunk,
                                 n_shards=world)
            t.shard.kind, t.shard.owner = "row_wise", None
            t.col_shards = None
        elif p.kind in ("table_wise", "data_parallel"):
            mine = p.kind == "data_parallel" or p.owner == rank
            w = _alloc_weight(rows if mine else 0, dim, device, shared and p.kind == "table_wise")
            if mine:
                _init_local(w, rows, seed * 1000 + ti * 64, init)
            t.weight = torch.nn.Parameter(w, requires_grad=False)
            t.shard = TableShard(name=t.name, rows=rows, dim=dim, weight=w, local_row0=0, chunk=rows, n_shards=1)
            t.shard.kind, t.shard.owner = p.kind, p.owner
            t.col_shards = None
        elif p.kind == "column_wise":
            cdim = dim // world
            w = _alloc_weight(rows, cdim, device, shared)
            _init_local(w, rows, seed * 1000 + ti * 64 + rank, init)
            t.weight = torch.nn.Parameter(w, requires_grad=False)
            shards = []
            for c in range(world):
                sw = w if c == rank else torch.zeros(0, cdim, device=device)
                s = TableShard(name=f"{t.name}#col{c}", rows=rows, dim=cdim, weight=sw, local_row0=0, chunk=rows,
                               n_shards=1)
                s.kind, s.owner = "column_wise", c
                shards.append(s)
            t.shard = shards[rank]
            t.col_shards = shards
        else:
            raise ValueError(f"unknown sharding kind {p.kind}")
        t.opt_state = []
    emb.sharded = True
    emb.rank, emb.world = rank, world
    if comm == "peer":
        emb.executor = PeerExecutor(emb, rank, world, device, group)
    else:
        emb.executor = A2AExecutor(rank, world, group)


# ---------------------------------------------------------------------------
# helpers shared by both executors
# ---------------------------------------------------------------------------

def _owner_of(t: TableShard, g: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    kind = getattr(t, "kind", "local")
    if kind == "row_wise":
        return torch.clamp(g // t.chunk, max=world - 1)
    if kind in ("table_wise", "column_wise"):
        return torch.full_like(g, t.owner)
    return torch.full_like(g, rank)


def _position_rows(spec: LookupSpec, i: int, ids: torch.Tensor, view: torch.Tensor):
    """Per-id (keys-to-keep mask, gradient rows) for slot i; pooled bags are
    expanded with 1/count (mean) and pad ids dropped."""
    sl = spec.slots[i]
    flat = ids.reshape(-1).long()
    if not sl.pool:
        return torch.ones_like(flat, dtype=torch.bool), view
    nb = view.shape[0]
    if sl.offsets is not None:
        lens = sl.offsets[1:] - sl.offsets[:-1]
        bag = torch.repeat_interleave(torch.arange(nb, device=flat.device), lens)
    else:
        bag = torch.arange(flat.numel(), device=flat.device) // max(flat.numel() // max(nb, 1), 1)
    keep = flat != sl.pad_id
    rows = view[bag].float()
    if sl.pool == 2:
        cnt = torch.zeros(nb, device=flat.device).index_add_(0, bag, keep.float())
        rows = rows / cnt.clamp_min(1)[bag].unsqueeze(-1)
    return keep, rows


# ---------------------------------------------------------------------------
# a2a baseline (NCCL / gloo collectives)
# ---------------------------------------------------------------------------

class A2AExecutor:
    """Collective exchange with the reference's program shape."""

    def __init__(self, rank: int, world: int, group=None):
        self.rank, self.world, self.group = rank, world, group
        self.comm_ms = 0.0

    def _a2a(self, x: torch.Tensor, send: list[int], recv: list[int]) -> torch.Tensor:
        out = x.new_empty((sum(recv),) + tuple(x.shape[1:]))
        dist.all_to_all_single(out, x.contiguous(), recv, send, group=self.group)
        return out

    def forward(self, spec: LookupSpec, ids: list[torch.Tensor], outs: list[torch.Tensor],
                backward: bool = False) -> None:
        spec.saved = {}
        for dim, sidx in _by_dim(spec).items():
            keys, owners, slot_of, gl = [], [], [], []
            for i in sidx:
                t = spec.tables[spec.slots[i].table]
                g = ids[i].reshape(-1).long()
                owners.append(_owner_of(t, g, self.world, self.rank))
                keys.append(g)
                slot_of.append(torch.full_like(g, i))
            keys, owners, slot_of = torch.cat(keys), torch.cat(owners), torch.cat(slot_of)
            tid = torch.tensor([spec.slots[i].table for i in sidx], device=keys.device)
            # table of each position, as an index into spec.tables
            table_of = torch.repeat_interleave(tid, torch.tensor([ids[i].numel() for i in sidx],
                                                                 device=keys.device))
            perm = torch.argsort(owners, stable=True)
            send = torch.bincount(owners, minlength=self.world)
            recv = torch.empty_like(send)
            dist.all_to_all_single(recv, send, group=self.group)
            send_l, recv_l = send.tolist(), recv.tolist()
            r_keys = self._a2a(keys[perm], send_l, recv_l)
            r_tab = self._a2a(table_of[perm], send_l, recv_l)
            rows = torch.zeros(r_keys.numel(), dim, dtype=torch.float32, device=keys.device)
            for ti in r_tab.unique().tolist():
                m = r_tab == ti
                rows[m] = _eager_rows(spec.tables[ti], r_keys[m])
            back = self._a2a(rows, recv_l, send_l)
            pos_rows = torch.empty_like(back)
            pos_rows[perm] = back
            off = 0
            for i in sidx:
                n = ids[i].numel()
                sl = spec.slots[i]
                view = _slot_view(outs[sl.group], sl.col, dim)
                pr = pos_rows[off:off + n]
                if sl.pool:
                    view.copy_(_pool_rows(pr, ids[i], sl, view.shape[0]))
                else:
                    view.copy_(pr.to(view.dtype))
                off += n
            spec.saved[dim] = (perm, send_l, recv_l, r_keys, r_tab)

    def backward(self, spec: LookupSpec, ids: list[torch.Tensor], grads: list[torch.Tensor], plan=None) -> None:
        for dim, sidx in _by_dim(spec).items():
            perm, send_l, recv_l, r_keys, r_tab = spec.saved[dim]
            rows, keep_all = [], []
            for i in sidx:
                sl = spec.slots[i]
                view = _slot_view(grads[sl.group], sl.col, dim)
                keep, r = _position_rows(spec, i, ids[i], view)
                rows.append(r.float() * keep.unsqueeze(-1))
                keep_all.append(keep)
            rows = torch.cat(rows)
            r_grads = self._a2a(rows[perm], send_l, recv_l)
            # positions that contribute nothing (pooled pad ids) must not reach
            # the optimizer at all: a zero gradient row would still take the
            # weight-decay step of row-wise Adagrad / Adam
            r_keep = self._a2a(torch.cat(keep_all)[perm].to(torch.uint8), send_l, recv_l).bool()
            dp_tables = []
            for ti in r_tab.unique().tolist():
                t = spec.tables[ti]
                if getattr(t, "kind", "local") == "data_parallel":
                    dp_tables.append(ti)
                    continue
                m = (r_tab == ti) & r_keep
                eager_sparse_update(t, spec.optimizer, r_keys[m], r_grads[m])
            # replicated tables: every rank applies everybody's rows
            all_dp = [ti for ti in sorted({spec.slots[i].table for i in sidx})
                      if getattr(spec.tables[ti], "kind", "local") == "data_parallel"]
            for ti in all_dp:
                m = (r_tab == ti) & r_keep
                k, gr = r_keys[m], r_grads[m]
                n = torch.tensor([k.numel()], device=k.device)
                ns = [torch.zeros_like(n) for _ in range(self.world)]
                dist.all_gather(ns, n, group=self.group)
                mx = int(max(x.item() for x in ns))
                kp = torch.full((mx,), -1, dtype=k.dtype, device=k.device)
                kp[:k.numel()] = k
                gp = torch.zeros(mx, dim, dtype=gr.dtype, device=gr.device)
                gp[:k.numel()] = gr
                ks = [torch.empty_like(kp) for _ in range(self.world)]
                gs = [torch.empty_like(gp) for _ in range(self.world)]
                dist.all_gather(ks, kp, group=self.group)
                dist.all_gather(gs, gp, group=self.group)
                K, G = torch.cat(ks), torch.cat(gs)
                valid = K >= 0
                eager_sparse_update(spec.tables[ti], spec.optimizer, K[valid], G[valid])


def _pool_rows(rows: torch.Tensor, ids: torch.Tensor, sl, n_bags: int) -> torch.Tensor:
    flat = ids.reshape(-1).long()
    if sl.offsets is not None:
        lens = sl.offsets[1:] - sl.offsets[:-1]
        bag = torch.repeat_interleave(torch.arange(n_bags, device=flat.device), lens)
    else:
        bag = torch.arange(flat.numel(), device=flat.device) // max(flat.numel() // max(n_bags, 1), 1)
    keep = (flat != sl.pad_id).unsqueeze(-1).to(rows.dtype)
    out = torch.zeros(n_bags, rows.shape[-1], dtype=rows.dtype, device=rows.device).index_add_(0, bag, rows * keep)
    if sl.pool == 2:
        cnt = torch.zeros(n_bags, dtype=rows.dtype, device=rows.device).index_add_(0, bag, keep.squeeze(-1))
        out = out / cnt.clamp_min(1).unsqueeze(-1)
    return out


# ---------------------------------------------------------------------------
# peer-memory product path
# ---------------------------------------------------------------------------

class SymmetricBuffer:
    """One device buffer per rank, mapped into every rank (CUDA IPC)."""

    def __init__(self, nbytes: int, device: torch.device, rank: int, world: int, group=None):
        self.rank, self.world, self.group = rank, world, group
        self.device = device
        self.opened: list[int] = []
        self.alloc(nbytes)

    def alloc(self, nbytes: int) -> None:
        C = _ext.core()
        self.close()
        self.nbytes = max(int(nbytes), 256)
        self.local = C.alloc_shared(self.nbytes, self.device.index)
        self.ptrs = exchange_pointers(self.local, self.rank, self.world, self.group, self.opened)

    def close(self) -> None:
        C = _ext.core()
        for b in self.opened:
            C.ipc_close(b)
        self.opened = []


def exchange_pointers(t: torch.Tensor, rank: int, world: int, group, opened: list[int]) -> list[int]:
    """All-gather IPC handles of ``t`` and map every peer's tensor; returns the
    per-rank addresses (this rank's own pointer for itself)."""
    C = _ext.core()
    h = C.ipc_handle(t) if t.numel() > 0 else torch.zeros(72, dtype=torch.uint8)
    hs = [None] * world
    dist.all_gather_object(hs, (h.numpy().tobytes(), t.numel() > 0), group=group)
    ptrs = []
    for r, (hb, valid) in enumerate(hs):
        if r == rank:
            ptrs.append(t.data_ptr())
        elif not valid:
            ptrs.append(0)
        else:
            addr, base = C.ipc_open(torch.frombuffer(bytearray(hb), dtype=torch.uint8))
            opened.append(base)
            ptrs.append(addr)
    return ptrs


_PLAN_DIMS = 8   # distinct embedding dims one lookup may route


class _DimPlan:
    """Backward routing of the slots of one embedding dim (see ``PeerExecutor._plan``)."""

    def __init__(self, dim, sidx, tables, weights, ptrs, tmeta, meta5, slot_ids, skeys, perm, seg, uniq, scale,
                 grow):
        self.dim, self.sidx, self.tables, self.weights, self.ptrs = dim, sidx, tables, weights, ptrs
        self.tmeta, self.meta5, self.slot_ids = tmeta, meta5, slot_ids
        self.skeys, self.perm, self.seg, self.uniq = skeys, perm, seg, uniq
        self.scale, self.grow = scale, grow


class _Plan:
    def __init__(self):
        self.dims: list[_DimPlan] = []
        self.host: torch.Tensor | None = None
        self.event: torch.cuda.Event | None = None


class PeerExecutor:
    def __init__(self, emb, rank: int, world: int, device: torch.device, group=None,
                 barrier_timeout_s: float = 30.0):
        self.rank, self.world, self.device, self.group = rank, world, device, group
        self.opened: list[int] = []
        self.timeout_ns = int(barrier_timeout_s * 1e9)
        self.epoch = 0
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.comm_ms = 0.0
        self.time_comm = False
        self._ev: list[tuple] = []
        # per-phase device timing of the backward (profiling aid; off by default)
        self.time_phases = os.environ.get("PD_EXCHANGE_PHASES", "0") == "1"
        self._phases: list[tuple[str, torch.cuda.Event]] = []
        self.phase_ms: dict[str, float] = {}
        # map every shard of every table
        for t in emb.tables():
            shards = t.col_shards if getattr(t, "col_shards", None) else [t.shard]
            for s in shards:
                kind = getattr(s, "kind", "local")
                if kind == "data_parallel":
                    continue
                if kind == "row_wise":
                    ptrs = exchange_pointers(s.weight, rank, world, group, self.opened)
                    s.peer_ptrs = torch.tensor(ptrs, dtype=torch.int64, device=device)
                else:  # whole table (or column block) on one owner
                    ptrs = exchange_pointers(s.weight, rank, world, group, self.opened)
                    s.peer_ptrs = torch.tensor([ptrs[s.owner]], dtype=torch.int64, device=device)
        self.pads = SymmetricBuffer(64 * 8, device, rank, world, group)
        self.pad_ptrs = torch.tensor(self.pads.ptrs, dtype=torch.int64)
        self.recv: dict[int, tuple[SymmetricBuffer, int]] = {}
        # routing plan of the backward, made during the forward on a side
        # stream: its own signal pads (epochs independent of the main
        # stream's barriers) and a count board int64 [W, _PLAN_DIMS * (W + 2)]
        self.plan_epoch = 0
        self.plan_row = _PLAN_DIMS * (world + 2)
        self.plan_buf = SymmetricBuffer(64 * 8 + world * self.plan_row * 8, device, rank, world, group)
        self.plan_pads = torch.tensor(self.plan_buf.ptrs, dtype=torch.int64)
        self.plan_boards = torch.tensor([p + 64 * 8 if p else 0 for p in self.plan_buf.ptrs], dtype=torch.int64)
        self.side = torch.cuda.Stream(device)
        self.barrier()

    # -- primitives --------------------------------------------------------
    def barrier(self) -> None:
        self.epoch += 1
        _ext.core().signal_barrier(self.pad_ptrs, self.rank, self.epoch, self.timeout_ns, self.err)

    def check(self) -> None:
        if int(self.err.item()) != 0:
            raise RuntimeError(f"peer embedding exchange error {int(self.err.item())} "
                               f"(2 = a peer did not arrive at the barrier in time)")

    def _recv_buffer(self, dim: int, cap_rows: int) -> tuple[int, list[int], list[int]]:
        """(capacity, key pointers, row pointers) of the receive slab for ``dim``."""
        cur = self.recv.get(dim)
        if cur is None or cur[1] < cap_rows:
            cap = max(int(cap_rows * 1.25), 1024)
            cap = (cap + 63) // 64 * 64  # keeps the fp32 row block 16-byte aligned after the int64 keys
            nbytes = cap * 8 + cap * dim * 4
            if cur is None:
                buf = SymmetricBuffer(nbytes, self.device, self.rank, self.world, self.group)
            else:
                buf = cur[0]
                buf.alloc(nbytes)
            self.recv[dim] = (buf, cap)
        buf, cap = self.recv[dim]
        kp = list(buf.ptrs)
        rp = [p + cap * 8 if p else 0 for p in buf.ptrs]
        return cap, kp, rp

    # -- lookup ------------------------------------------------------------
    def forward(self, spec: LookupSpec, ids: list[torch.Tensor], outs: list[torch.Tensor],
                backward: bool = False) -> "_Plan | None":
        """Gather every slot from the owners' shards (peer loads).

        Unpooled lookups are planned first -- keys sorted by owner and row,
        unique segments -- and gathered once per unique row in address order,
        then expanded to every position.  With ``backward`` the plan is kept
        for the backward and its per-owner counts are exchanged on a side
        stream that overlaps the rest of the forward.  Pooled lookups use the
        direct gather and plan on the side stream."""
        ev = self._event_pair()
        if any(sl.pool for sl in spec.slots):
            _native_forward(spec, ids, outs)
            self._event_end(ev)
            if not backward:
                return None
            main = torch.cuda.current_stream(self.device)
            self.side.wait_stream(main)
            with torch.cuda.stream(self.side):
                plan = self._plan_core(spec, ids, outs)
            for t in ids:
                t.record_stream(self.side)
            for d in plan.dims:          # made on the side stream, read by the backward on this one
                for t in (d.skeys, d.perm, d.seg, d.uniq, d.scale, d.grow):
                    if t is not None:
                        t.record_stream(main)
            self._plan_counts(plan, main)
            return plan
        C = _ext.core()
        plan = self._plan_core(spec, ids, outs)
        for d in plan.dims:
            views = [_slot_view(outs[spec.slots[i].group], spec.slots[i].col, d.dim) for i in d.sidx]
            C.emb_gather_planned(d.slot_ids, views, d.meta5[:, :4].contiguous(), d.weights, d.ptrs, d.tmeta, d.dim,
                                 d.skeys, d.perm, d.seg, d.uniq, spec.err)
        self._event_end(ev)
        if not backward:
            return None
        self._plan_counts(plan, torch.cuda.current_stream(self.device))
        return plan

    def _plan_core(self, spec: LookupSpec, ids: list[torch.Tensor], outs: list[torch.Tensor]) -> "_Plan":
        """Per embedding dim, on the current stream: owner-sorted keys, their
        permutation, the unique-row segment of every sorted key and the key of
        every unique segment.  Needs the ids only (``outs`` give the shapes)."""
        C = _ext.core()
        W = self.world
        groups = list(_by_dim(spec).items())
        if len(groups) > _PLAN_DIMS:
            raise RuntimeError(f"peer exchange plans at most {_PLAN_DIMS} embedding dims, got {len(groups)}")
        plan = _Plan()
        for dim, sidx in groups:
            tables, remap = _launch_tables(spec, sidx)
            weights = [t.weight for t in tables]
            ptrs = [t.device_ptrs() for t in tables]
            tmeta = _table_meta(tables)
            slot_ids = [ids[i].reshape(-1) for i in sidx]
            views, meta4, offs, any_pooled = [], [], [], False
            for i in sidx:
                sl = spec.slots[i]
                views.append(_slot_view(outs[sl.group], sl.col, dim))
                L = 0
                if sl.pool:
                    any_pooled = True
                    nb = outs[sl.group].numel() // outs[sl.group].shape[-1]
                    L = ids[i].numel() // max(nb, 1) if sl.offsets is None else 0
                meta4.append([remap[sl.table], sl.pool, L, sl.pad_id])
                offs.append(sl.offsets if sl.offsets is not None else ids[i].new_empty(0, dtype=torch.int64))
            meta4 = torch.tensor(meta4, dtype=torch.int64)
            keys = C.emb_keys(slot_ids, views, meta4, offs, weights, ptrs, tmeta, dim)
            ometa = torch.tensor([[int(tmeta[k, 2]), t.chunk, _KIND_CODE.get(getattr(t, "kind", "row_wise"), 0),
                                   t.owner if getattr(t, "owner", None) is not None else 0]
                                  for k, t in enumerate(tables)], dtype=torch.int64)
            skeys, perm = torch.sort(C.owner_keys(keys, ometa, W))
            n = skeys.numel()
            first = torch.ones(n, dtype=torch.bool, device=self.device)
            if n > 1:
                torch.ne(skeys[1:], skeys[:-1], out=first[1:])
            seg = torch.cumsum(first, 0) - 1
            uniq = torch.empty(n, dtype=torch.int64, device=self.device).scatter_(0, seg, skeys & _KEY_MASK)
            scale = grow = None
            if any_pooled:
                scale, grow = C.emb_pooled_scale(slot_ids, views, meta4, offs, weights, ptrs, tmeta, dim)
            meta5 = torch.cat([meta4, torch.tensor([[x.numel()] for x in slot_ids], dtype=torch.int64)], 1)
            plan.dims.append(_DimPlan(dim, sidx, tables, weights, ptrs, tmeta, meta5, slot_ids, skeys, perm, seg,
                                      uniq, scale, grow))
        return plan

    def _plan_counts(self, plan: "_Plan", main) -> None:
        """Per-owner unique counts of every rank, on the side stream: counted
        from the sorted keys (owner boundaries by binary search, no atomics),
        written into every rank's board with peer stores, published by a
        signal barrier and copied to pinned host memory.  The backward waits
        on this plan's event, which completed long before, instead of
        synchronising the host with the compute stream."""
        C = _ext.core()
        W = self.world
        side = self.side
        side.wait_stream(main)
        with torch.cuda.stream(side):
            row = torch.zeros(self.plan_row, dtype=torch.int64, device=self.device)
            bounds = torch.arange(W + 2, dtype=torch.int64, device=self.device) << _OWNER_SHIFT
            for di, d in enumerate(plan.dims):
                n = d.skeys.numel()
                if n == 0:
                    continue
                # owner W = replicated tables, W + 1 = padding keys (dropped)
                pos = torch.searchsorted(d.skeys, bounds)
                before = torch.where(pos > 0, d.seg[(pos - 1).clamp_(min=0)] + 1, torch.zeros_like(pos))
                cnt = torch.diff(torch.cat([before, d.seg[-1:] + 1]))
                row[di * (W + 2): (di + 1) * (W + 2)] = cnt
            C.peer_put_row(row, self.plan_boards, self.rank)
            self.plan_epoch += 1
            C.signal_barrier(self.plan_pads, self.rank, self.plan_epoch, self.timeout_ns, self.err)
            board = self.plan_buf.local[64 * 8:].view(torch.int64)[: W * self.plan_row]
            plan.host = torch.empty(W * self.plan_row, dtype=torch.int64, pin_memory=True)
            plan.host.copy_(board, non_blocking=True)
            plan.event = torch.cuda.Event()
            plan.event.record(side)
        for d in plan.dims:
            for t in (d.skeys, d.seg):
                t.record_stream(side)

    def _mark(self, name: str) -> None:
        if self.time_phases:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._phases.append((name, e))

    def take_phase_ms(self) -> dict[str, float]:
        """Accumulated device time per backward phase (syncs)."""
        if self._phases:
            torch.cuda.synchronize()
            for (_, a), (name, b) in zip(self._phases[:-1], self._phases[1:]):
                self.phase_ms[name] = self.phase_ms.get(name, 0.0) + a.elapsed_time(b)
            self._phases = []
        return dict(self.phase_ms)

    def backward(self, spec: LookupSpec, ids: list[torch.Tensor], grads: list[torch.Tensor],
                 plan: "_Plan | None" = None) -> None:
        """Local reduction per unique row, push to the owners, owner update.
        Without a plan from the forward (a lookup run outside autograd) the
        plan is made here."""
        if plan is None:
            plan = self._plan_core(spec, ids, grads)
            self._plan_counts(plan, torch.cuda.current_stream(self.device))
        ev = self._event_pair()
        self._mark("start")
        C = _ext.core()
        opt = spec.optimizer
        bc1, bc2 = opt.bias_corrections()
        W = self.world
        main = torch.cuda.current_stream(self.device)
        main.wait_event(plan.event)
        plan.event.synchronize()                  # finished during the forward: no drain of the compute stream
        board = plan.host.view(W, self.plan_row)
        for di, d in enumerate(plan.dims):
            dim = d.dim
            M = board[:, di * (W + 2): di * (W + 2) + W + 1]   # [src, owner 0..W] unique counts
            U = int(M[self.rank].sum())
            views = [_slot_view(grads[spec.slots[i].group], spec.slots[i].col, dim) for i in d.sidx]
            reduced = torch.empty(U + 1, dim, dtype=torch.float32, device=self.device)  # + the padding run
            C.emb_reduce_update(views, d.meta5, d.weights, d.ptrs, [w.new_empty(0) for w in d.weights],
                                [w.new_empty(0) for w in d.weights], d.tmeta, dim, d.skeys, d.perm, d.scale,
                                d.grow, 0, 0.0, 0.0, 0.0, 0.0, 0.0, 1.0, 1.0, self.err, out_rows=reduced, seg=d.seg)
            self._mark("local_reduce")
            col = M.sum(0)
            need = [int(col[o] + col[W]) for o in range(W)]
            cap, kp, rp = self._recv_buffer(dim, max(need))
            dst_off = [int(M[: self.rank, o].sum()) for o in range(W)]
            bcast_off = [int(col[o] + M[: self.rank, W].sum()) for o in range(W)]
            seg_start = [0] + torch.cumsum(M[self.rank], 0).tolist()
            C.push_rows(d.uniq[:U], reduced[:U], torch.tensor(kp), torch.tensor(rp),
                        torch.tensor(dst_off), torch.tensor(bcast_off), torch.tensor(seg_start))
            self._mark("push")
            self.barrier()
            self._mark("barrier")
            R = need[self.rank]
            if R:
                buf, cap = self.recv[dim]
                rk = buf.local[: cap * 8].view(torch.int64)[:R]
                rr = buf.local[cap * 8: cap * 8 + cap * dim * 4].view(torch.float32).view(cap, dim)[:R]
                sk2, perm2 = torch.sort(rk)
                self._mark("owner_sort")
                s1 = [t.state[0] if len(t.state) > 0 else t.weight.new_empty(0) for t in d.tables]
                s2 = [t.state[1] if len(t.state) > 1 else t.weight.new_empty(0) for t in d.tables]
                meta_r = torch.tensor([[0, 0, 0, -1, R]], dtype=torch.int64)
                C.emb_reduce_update([rr], meta_r, d.weights, d.ptrs, s1, s2, d.tmeta, dim, sk2, perm2, None, None,
                                    opt.code, opt.lr * opt.lr_scale, opt.eps, opt.weight_decay, opt.beta1,
                                    opt.beta2, bc1, bc2, self.err)
                self._mark("owner_update")
        self.barrier()
        self._mark("final_barrier")
        self._event_end(ev)

    # -- timing ------------------------------------------------------------
    def _event_pair(self):
        if not self.time_comm:
            return None
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        return (a, b)

    def _event_end(self, ev) -> None:
        if ev is not None:
            ev[1].record()
            self._ev.append(ev)

    def take_comm_ms(self) -> float:
        """Device time spent in lookup + exchange since the last call (syncs)."""
        if self._ev:
            torch.cuda.synchronize()
            self.comm_ms = sum(a.elapsed_time(b) for a, b in self._ev)
            self._ev = []
        else:
            self.comm_ms = 0.0
        return self.comm_ms

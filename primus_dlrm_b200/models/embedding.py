"""Embedding tables (unpooled collection + pooled bag collection).

Same module tree and state-dict keys as the reference's TorchRec wrapper
(``primus_dlrm/models/embedding.py:72-175``):

* ``emb.ec.embeddings.<table>.weight``      -- unpooled tables (pooling "none")
* ``emb.ebc.embedding_bags.<table>.weight`` -- pooled tables (mean / sum)

Differences (B200-native): no TorchRec/KJT.  ``Embeddings.lookup_groups``
gathers many features in one kernel launch straight into concatenated,
compute-dtype group buffers; the optimizer runs inside the backward
(``primus_dlrm_b200.ops.embedding``).  Pooled lookups exclude the padding id
(0), matching ``_build_pooled_kjt`` (``primus_dlrm/models/embedding.py:179-204``).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from primus_dlrm_b200.config import EmbeddingTableConfig
from primus_dlrm_b200.ops import _ext
from primus_dlrm_b200.ops.embedding import (
    LookupSpec, Slot, SparseOptimizer, TableShard, grouped_lookup,
)

_POOL = {"none": 0, "sum": 1, "mean": 2}


def init_table_(w: torch.Tensor, rows: int, how: str, generator: torch.Generator | None = None) -> None:
    """TorchRec default: U(-sqrt(1/rows), sqrt(1/rows)); ``normal``: N(0, 1)."""
    if how == "normal":
        w.normal_(0.0, 1.0, generator=generator)
    else:
        b = math.sqrt(1.0 / max(rows, 1))
        w.uniform_(-b, b, generator=generator)


class Table(nn.Module):
    """One table (or this rank's row shard of it). ``weight`` is updated by the
    fused optimizer inside the lookup backward, never by autograd."""

    def __init__(self, cfg: EmbeddingTableConfig, device, init: str = "uniform",
                 local_row0: int = 0, local_rows: int | None = None):
        super().__init__()
        self.name = cfg.name
        self.num_embeddings = cfg.num_embeddings
        self.embedding_dim = cfg.embedding_dim
        self.pooling = cfg.pooling
        self.features = list(cfg.features)
        local_rows = cfg.num_embeddings if local_rows is None else local_rows
        w = torch.empty(local_rows, cfg.embedding_dim, device=device, dtype=torch.float32)
        if w.device.type != "meta":
            init_table_(w, cfg.num_embeddings, init)
        self.weight = nn.Parameter(w, requires_grad=False)
        self.shard = TableShard(name=cfg.name, rows=cfg.num_embeddings, dim=cfg.embedding_dim,
                                weight=self.weight.data, local_row0=local_row0)
        self.col_shards: list[TableShard] | None = None  # column-wise sharding: one shard per rank
        self.opt_state: list[torch.Tensor] = []

    def lookup_shards(self) -> list[tuple[TableShard, int]]:
        """(shard, column offset) pairs that make up one feature's embedding."""
        if self.col_shards:
            return [(s, c * s.dim) for c, s in enumerate(self.col_shards)]
        return [(self.shard, 0)]

    def ensure_state(self, opt: SparseOptimizer) -> None:
        """Optimizer state for the locally stored rows (allocated on first use)."""
        if self.weight.device.type == "meta":
            return
        shapes = opt.state_shapes(self.weight.shape[0], self.weight.shape[1])
        if len(self.opt_state) != len(shapes) or any(
                s.device != self.weight.device or tuple(s.shape) != sh for s, sh in zip(self.opt_state, shapes)):
            self.opt_state = [torch.zeros(sh, dtype=torch.float32, device=self.weight.device) for sh in shapes]
        local = self.shard
        local.weight = self.weight.data
        local.state = self.opt_state

    def _apply(self, fn, recurse=True):
        out = super()._apply(fn, recurse)
        self.shard.weight = self.weight.data
        self.opt_state = [fn(s) for s in self.opt_state]
        self.shard.state = self.opt_state
        return out


class EmbeddingCollection(nn.Module):
    def __init__(self, tables: list[EmbeddingTableConfig], device, init: str):
        super().__init__()
        self.embeddings = nn.ModuleDict({t.name: Table(t, device, init) for t in tables})


class EmbeddingBagCollection(nn.Module):
    def __init__(self, tables: list[EmbeddingTableConfig], device, init: str):
        super().__init__()
        self.embedding_bags = nn.ModuleDict({t.name: Table(t, device, init) for t in tables})


class Embeddings(nn.Module):
    """Pooled + unpooled tables behind one lookup API.

    ``forward({feature: ids})`` -> ``{feature: emb}`` is the reference API
    (``[B]`` -> ``[B, D]``, ``[B, L]`` -> ``[B, L, D]`` unpooled or ``[B, D]``
    pooled).  ``lookup_groups`` is the fused API used by the models.
    """

    def __init__(self, table_specs: list[EmbeddingTableConfig], device=None, embedding_init: str = "uniform",
                 scalar_feature_names: set[str] | None = None, optimizer: SparseOptimizer | None = None):
        super().__init__()
        device = torch.device("cpu") if device is None else torch.device(device)
        pooled = [t for t in table_specs if t.pooling in ("mean", "sum")]
        unpooled = [t for t in table_specs if t.pooling not in ("mean", "sum")]
        self.ec = EmbeddingCollection(unpooled, device, embedding_init) if unpooled else None
        self.ebc = EmbeddingBagCollection(pooled, device, embedding_init) if pooled else None
        self._feature_table: dict[str, Table] = {}
        self._feature_dims: dict[str, int] = {}
        for coll in (self.ec, self.ebc):
            if coll is None:
                continue
            tables = coll.embeddings if coll is self.ec else coll.embedding_bags
            for t in tables.values():
                for f in t.features:
                    self._feature_table[f] = t
                    self._feature_dims[f] = t.embedding_dim
        self._scalar_features = set(scalar_feature_names or ()) & set(self._feature_table)
        self.optimizer = optimizer or SparseOptimizer()
        self.padding_idx = 0
        self._anchor: torch.Tensor | None = None
        self.err = None
        self.native = True  # set False to force the eager oracle path
        self.executor = None  # set by parallel.sharded_embedding.shard_embeddings
        self.sharded = False

    # -- bookkeeping -------------------------------------------------------
    def tables(self) -> list[Table]:
        out = []
        if self.ec is not None:
            out.extend(self.ec.embeddings.values())
        if self.ebc is not None:
            out.extend(self.ebc.embedding_bags.values())
        return out

    def feature_dim(self, f: str) -> int:
        return self._feature_dims[f]

    def is_pooled(self, f: str) -> bool:
        return self._feature_table[f].pooling in ("mean", "sum")

    def _grad_anchor(self, device) -> torch.Tensor:
        if self._anchor is None or self._anchor.device != device:
            self._anchor = torch.zeros((), device=device, requires_grad=True)
        return self._anchor

    def error_word(self, device) -> torch.Tensor:
        if self.err is None or self.err.device != device:
            self.err = torch.zeros(1, dtype=torch.int32, device=device)
        return self.err

    def check_errors(self) -> None:
        """Raise if a kernel recorded an out-of-range id (host sync)."""
        if self.err is not None and int(self.err.item()) != 0:
            code = int(self.err.item())
            self.err.zero_()
            raise RuntimeError(f"embedding kernel error code {code} (1 = id out of range)")

    # -- lookups -----------------------------------------------------------
    def lookup_groups(self, features: dict[str, torch.Tensor], groups: list[list[str]],
                      dtype: torch.dtype = torch.float32,
                      offsets: dict[str, torch.Tensor] | None = None) -> list[torch.Tensor]:
        """Gather each group's features concatenated along the last dim.

        All features of a group must share the leading shape: ``ids.shape``
        for unpooled features, ``ids.shape[:-1]`` (or the bag count given by
        ``offsets``) for pooled ones.
        """
        tables: list[TableShard] = []
        tindex: dict[int, int] = {}
        slots: list[Slot] = []
        ids: list[torch.Tensor] = []
        shapes: list[tuple[int, ...]] = []
        device = None
        for gi, group in enumerate(groups):
            col = 0
            lead = None
            for f in group:
                t = self._feature_table[f]
                t.ensure_state(self.optimizer)
                x = features[f]
                device = x.device
                pool = _POOL.get(t.pooling, 0)
                off = offsets.get(f) if offsets else None
                if pool:
                    this_lead = (off.numel() - 1,) if off is not None else tuple(x.shape[:-1])
                else:
                    this_lead = tuple(x.shape)
                if lead is None:
                    lead = this_lead
                elif lead != this_lead:
                    raise ValueError(f"group {group}: feature {f} has leading shape {this_lead}, expected {lead}")
                for shard, coff in t.lookup_shards():
                    if id(shard) not in tindex:
                        tindex[id(shard)] = len(tables)
                        tables.append(shard)
                    slots.append(Slot(table=tindex[id(shard)], group=gi, col=col + coff, pool=pool,
                                      pad_id=self.padding_idx if pool else -1, offsets=off))
                    ids.append(x if x.is_contiguous() else x.contiguous())
                col += t.embedding_dim
            shapes.append(tuple(lead) + (col,))
        native = (self.native and device is not None and device.type == "cuda"
                  and _ext.native_enabled(device))
        executor = self.executor
        if native:
            ids = [i if i.dtype in (torch.int32, torch.int64) else i.long() for i in ids]
            if len({i.dtype for i in ids}) > 1:
                ids = [i.long() for i in ids]
        spec = LookupSpec(tables=tables, slots=slots, group_shapes=shapes, dtype=dtype,
                          optimizer=self.optimizer, native=native,
                          err=self.error_word(device) if (native or executor is not None) else None,
                          executor=executor)
        return grouped_lookup(spec, ids, self._grad_anchor(device))

    def forward(self, features: dict[str, torch.Tensor], padding_idx: int = 0) -> dict[str, torch.Tensor]:
        names = [f for f in features if f in self._feature_table]
        outs = self.lookup_groups({f: features[f] for f in names}, [[f] for f in names])
        return dict(zip(names, outs))

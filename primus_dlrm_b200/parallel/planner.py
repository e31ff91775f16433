"""Embedding sharding plan.

Per-table sharding choice with the reference's precedence
(``primus_dlrm/distributed/wrapper.py:277-379``): inline table spec >
``embedding_sharding.default_table_sharding`` > the global
``embedding_sharding.strategy`` (``auto`` = no constraint).  Topology caps
come from the environment (``PRIMUS_TORCHREC_HBM_CAP_GB``, ``_DDR_CAP_GB``,
``_LOCAL_WORLD_SIZE``) before the YAML ``topology`` block
(``wrapper.py:437-469``).

``auto`` is decided here with a rule fitted to the NVLink pull/push design:
a row-wise table spreads both its bytes and its lookup traffic evenly over
all GPUs, so every table too large to replicate cheaply is row-wise;
mid-size tables are placed whole on the least-loaded rank (table-wise) when
they fit its HBM budget; tiny tables are replicated (data-parallel).
``plan_sharding`` also recommends DDP vs FSDP for the dense part with the
reference heuristic (``primus_dlrm/distributed/planner.py:54-161``): FSDP
once dense params + Adam state exceed 10% of HBM.
"""
from __future__ import annotations

import logging
import os
from dataclasses import dataclass, field

from primus_dlrm_b200.config import Config, EmbeddingTableConfig, TableShardingSpec

logger = logging.getLogger(__name__)

KINDS = ("row_wise", "table_wise", "column_wise", "data_parallel")
_EXTRA_FIELDS = ("compute_kernel", "cache_load_factor", "min_partition", "enforce_hbm", "output_dtype", "ranks")

# bytes of optimizer state per fp32 weight byte (Adam m+v)
_OPT_MULT = {"adam": 3.0, "row_wise_adagrad": 1.0, "adagrad": 2.0, "sgd": 1.0}


@dataclass
class TablePlan:
    name: str
    kind: str                     # row_wise | table_wise | column_wise | data_parallel
    owner: int | None = None      # table_wise owner rank
    ranks: list[int] = field(default_factory=list)
    compute_kernel: str = "fused"
    output_dtype: str | None = None
    reason: str = ""


@dataclass
class Topology:
    world_size: int
    hbm_cap_gb: float = 161.0      # ~90% of a B200's 178 GiB
    ddr_cap_gb: float | None = None
    local_world_size: int = 8


def merge_sharding_specs(inline: TableShardingSpec | None, default: TableShardingSpec | None,
                         global_strategy: str) -> TableShardingSpec | None:
    """Field-by-field merge (inline wins, then default; the global strategy only
    supplies ``sharding_type``).  ``None`` = nothing constrained (auto)."""
    st = None
    if inline is not None and inline.sharding_type is not None:
        st = inline.sharding_type
    elif default is not None and default.sharding_type is not None:
        st = default.sharding_type
    elif global_strategy not in ("auto", None):
        st = global_strategy
    specs = [s for s in (inline, default) if s is not None]
    extra = any(getattr(s, n) is not None for s in specs for n in _EXTRA_FIELDS)
    if st is None and not extra:
        return None

    def pick(n):
        for s in (inline, default):
            if s is not None and getattr(s, n) is not None:
                return getattr(s, n)
        return None

    return TableShardingSpec(sharding_type=st, **{n: pick(n) for n in _EXTRA_FIELDS})


def build_topology(config: Config, world_size: int) -> Topology:
    topo = config.distributed.embedding_sharding.topology

    def env(name):
        v = os.environ.get(name)
        return v.strip() if v and v.strip() else None

    hbm = env("PRIMUS_TORCHREC_HBM_CAP_GB")
    ddr = env("PRIMUS_TORCHREC_DDR_CAP_GB")
    lws = env("PRIMUS_TORCHREC_LOCAL_WORLD_SIZE")
    t = Topology(world_size=world_size)
    if hbm is not None:
        t.hbm_cap_gb = float(hbm)
    elif topo.hbm_cap_gb is not None:
        t.hbm_cap_gb = float(topo.hbm_cap_gb)
    if ddr is not None:
        t.ddr_cap_gb = float(ddr)
    elif topo.ddr_cap_gb is not None:
        t.ddr_cap_gb = float(topo.ddr_cap_gb)
    if lws is not None:
        t.local_world_size = int(lws)
    elif topo.local_world_size is not None:
        t.local_world_size = int(topo.local_world_size)
    return t


def plan_tables(config: Config, world_size: int, topology: Topology | None = None) -> dict[str, TablePlan]:
    """Sharding decision for every (resolved) embedding table."""
    topology = topology or build_topology(config, world_size)
    es = config.distributed.embedding_sharding
    strategy = es.strategy if es.strategy in KINDS + ("auto",) else "auto"
    if es.strategy not in KINDS + ("auto",):
        logger.warning("unknown global sharding strategy %r; falling back to auto", es.strategy)
    opt_mult = _OPT_MULT.get(config.train.embedding_optimizer, 3.0)
    budget = topology.hbm_cap_gb * 1e9 * 0.5  # embedding share of HBM per rank
    load = [0.0] * world_size
    plans: dict[str, TablePlan] = {}
    tables = sorted(config.model.resolved_embedding_tables(), key=lambda t: -t.num_embeddings * t.embedding_dim)
    for t in tables:
        spec = merge_sharding_specs(t.sharding, es.default_table_sharding, strategy)
        nbytes = t.num_embeddings * t.embedding_dim * 4 * (1 + opt_mult)
        kind = spec.sharding_type if spec is not None and spec.sharding_type else None
        if kind is not None and kind not in KINDS:
            logger.warning("unknown sharding_type %r for %s; using auto", kind, t.name)
            kind = None
        reason = "constrained" if kind else ""
        if world_size <= 1:
            kind, reason = "data_parallel", "single rank"
        elif kind is None:
            if nbytes >= 256e6 or nbytes > budget:
                kind, reason = "row_wise", f"{nbytes / 1e9:.2f} GB with optimizer state"
            elif nbytes >= 4e6:
                kind, reason = "table_wise", f"mid-size ({nbytes / 1e6:.1f} MB)"
            else:
                kind, reason = "data_parallel", f"tiny ({nbytes / 1e3:.0f} KB)"
        if kind == "column_wise" and t.embedding_dim % (4 * world_size) != 0:
            logger.warning("%s: dim %d does not split into %d column shards of a multiple of 4; row_wise",
                           t.name, t.embedding_dim, world_size)
            kind = "row_wise"
        p = TablePlan(name=t.name, kind=kind, reason=reason)
        if spec is not None:
            p.compute_kernel = spec.compute_kernel or "fused"
            p.output_dtype = spec.output_dtype
        if kind == "table_wise":
            if spec is not None and spec.ranks:
                p.owner = int(spec.ranks[0]) % world_size
            else:
                p.owner = min(range(world_size), key=lambda r: load[r])
            load[p.owner] += nbytes
        elif kind == "row_wise":
            for r in range(world_size):
                load[r] += nbytes / world_size
        elif kind == "column_wise":
            for r in range(world_size):
                load[r] += nbytes / world_size
        else:
            for r in range(world_size):
                load[r] += nbytes
        p.ranks = list(range(world_size)) if kind != "table_wise" else [p.owner]
        plans[t.name] = p
    return plans


def recommend_dense_strategy(dense_params: int, topology: Topology) -> str:
    return "fsdp" if dense_params * 4 * 3 > topology.hbm_cap_gb * 1e9 * 0.1 else "ddp"


def log_plan(plans: dict[str, TablePlan]) -> None:
    for p in plans.values():
        where = f"rank {p.owner}" if p.kind == "table_wise" else f"{len(p.ranks)} ranks"
        logger.info("  Shard: %s -> type=%s (%s) %s", p.name, p.kind, where, p.reason)

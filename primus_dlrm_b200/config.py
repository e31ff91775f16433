"""YAML configuration schema.

The schema (section names, field names, defaults, load-time semantics) is a
public contract shared with Primus-DLRM configs, so every reference YAML in
``configs/`` loads unchanged.  Reference: ``primus_dlrm/config.py:1-831``.

Differences from the reference are additive only:

* ``DataConfig.history_lengths`` -- per sequence-group history length
  (the v6 and ~5B benchmark configs use pools of 512/128/256).
* ``SyntheticDataConfig`` -- Zipf id sampling, per-task Bernoulli rates,
  regression labels, dense-feature distributions, log-uniform table sizes.
* ``TransformerConfig.norm`` -- ``rmsnorm`` (reference) or ``layernorm``.
* ``ModelConfig.dcn_low_rank`` / ``ModelConfig.dlrm_layout`` -- low-rank
  DCNv2 cross layers and a Criteo-style single-tower DLRM.
* ``TrainConfig.kernels`` -- ``native`` (sm_100a kernels) or ``eager``
  (plain PyTorch semantics, the oracle), ``eval_num_candidates``.
* ``DistributedConfig.comm`` -- ``peer`` (NVLink peer-memory kernels) or
  ``nccl`` (the NCCL baseline).

Loading is type-hint driven: nested dataclasses, ``Optional[...]`` and
``list[Dataclass]`` fields are instantiated recursively; unknown keys are
ignored (``primus_dlrm/config.py:792-794``).
"""
from __future__ import annotations

import dataclasses
import typing
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any, Optional, Union

import yaml


# ---------------------------------------------------------------------------
# data
# ---------------------------------------------------------------------------

@dataclass
class SchemaConfig:
    """Batch-key -> embedding-feature mapping and KJT feature order."""
    batch_to_feature: dict[str, str] = field(default_factory=dict)
    kjt_feature_order: list[str] = field(default_factory=list)


@dataclass
class SyntheticDataConfig:
    """Synthetic data generator (``primus_dlrm/config.py:274-297``) plus the
    benchmark extensions (distribution knobs)."""
    enabled: bool = False
    seed: int = 42
    num_samples: int = 100_000
    num_prebatched: int = 16
    label_positive_rate: float = 0.3
    sparse_id_min: int = 0
    sparse_id_max: int = 0
    sparse_len_min: int = 0
    sparse_len_max: int = 0
    # --- additive ---
    # "uniform" (reference) or "zipf"
    id_distribution: str = "uniform"
    zipf_alpha: float = 1.05
    # per-task Bernoulli rate; tasks absent here use label_positive_rate
    task_positive_rates: dict[str, float] = field(default_factory=dict)
    # dense feature distribution: "uniform" (reference), "normal", "lognormal"
    dense_distribution: str = "uniform"


@dataclass
class DataConfig:
    """Dataset / preprocessing configuration (``primus_dlrm/config.py:10-61``)."""
    dataset_size: str = "50m"
    history_length: int = 20
    history_mode: str = "last_l"
    history_days: int = 30
    num_negatives: int = 0
    negative_sampler: str = "none"
    session_gap_seconds: int = 1800
    num_workers: int = 4
    prefetch_factor: int = 2
    enable_counters: bool = False
    counter_windows_days: list[int] = field(default_factory=lambda: [30])
    data_dir: str = "data"
    use_cache: bool = True
    synthetic: SyntheticDataConfig = field(default_factory=SyntheticDataConfig)
    schema: Union[SchemaConfig, str] = field(default_factory=SchemaConfig)
    # --- additive: per sequence-group history length (group -> L) ---
    history_lengths: dict[str, int] = field(default_factory=dict)

    def group_length(self, group: str) -> int:
        return int(self.history_lengths.get(group, self.history_length))


# ---------------------------------------------------------------------------
# features / model
# ---------------------------------------------------------------------------

@dataclass
class TableShardingSpec:
    """Per-table sharding constraints (``primus_dlrm/config.py:68-98``).

    ``sharding_type``: row_wise | table_wise | column_wise | data_parallel.
    ``compute_kernel``: fused | fused_uvm | fused_uvm_caching | dense -- the
    native sharder keeps every table in HBM (``fused``); the UVM variants
    place the table in pinned host memory mapped into the device.
    ``ranks`` pins a table-wise table to a rank.
    """
    sharding_type: Optional[str] = None
    compute_kernel: Optional[str] = None
    cache_load_factor: Optional[float] = None
    min_partition: Optional[int] = None
    enforce_hbm: Optional[bool] = None
    output_dtype: Optional[str] = None
    ranks: Optional[list[int]] = None


@dataclass
class EmbeddingTableConfig:
    name: str = ""
    features: list[str] = field(default_factory=list)
    num_embeddings: int = 0
    embedding_dim: int = 0
    pooling: str = "none"
    sharding: Optional[TableShardingSpec] = None


CROSS_FEATURE_KEYS = ("uid", "item_id", "artist_id", "album_id", "hour_of_day", "is_organic")


@dataclass
class CrossFeatureSpec:
    """Hashed cross-product table, auto-registered at load time
    (``primus_dlrm/config.py:123-166``)."""
    name: str = ""
    keys: list[str] = field(default_factory=list)
    num_embeddings: int = 0
    salt: int = 0
    enabled: bool = True
    sharding: Optional[TableShardingSpec] = None


TOWER_USER = "user"
TOWER_ITEM = "item"


class _Tower:
    """DLRM tower routing: "" = both towers, "user", or "item"."""
    tower: str = ""

    def in_user_tower(self) -> bool:
        return self.tower != TOWER_ITEM

    def in_item_tower(self) -> bool:
        return self.tower != TOWER_USER


@dataclass
class ScalarFeatureSpec(_Tower):
    name: str = ""
    tower: str = ""


@dataclass
class DenseFeatureSpec(_Tower):
    name: str = ""
    dim: int = 0
    value_range_min: float = 0.0
    value_range_max: float = 1.0
    project: bool = True
    activation: str = "gelu"
    tower: str = ""


@dataclass
class FeatureConfig:
    sequence_groups: dict[str, list[str]] = field(default_factory=dict)
    scalar_features: list[ScalarFeatureSpec] = field(default_factory=list)
    dense_features: list[DenseFeatureSpec] = field(default_factory=list)

    def __post_init__(self):
        self.scalar_features = [
            ScalarFeatureSpec(name=s) if isinstance(s, str) else s
            for s in self.scalar_features
        ]

    @property
    def scalar_feature_names(self) -> list[str]:
        return [s.name for s in self.scalar_features]

    @property
    def user_scalar_features(self) -> list[ScalarFeatureSpec]:
        return [s for s in self.scalar_features if s.in_user_tower()]

    @property
    def item_scalar_features(self) -> list[ScalarFeatureSpec]:
        return [s for s in self.scalar_features if s.in_item_tower()]

    def all_ec_feature_names(self) -> list[str]:
        """Scalars first, then sequence features group by group."""
        out = list(self.scalar_feature_names)
        for feats in self.sequence_groups.values():
            out.extend(feats)
        return out


@dataclass
class TransformerConfig:
    d_model: int = 128
    n_heads: int = 4
    n_layers: int = 4
    ffn_mult: int = 4
    n_ns_tokens: int = 8
    use_pyramid: bool = True
    dropout: float = 0.1
    pos_embed: bool = True
    # The reference accepts sdpa | fav2 | fav4 | turbo.  Here "native" is the
    # sm_100a pyramid attention kernel; every other value maps onto it when
    # the native kernels are enabled and onto SDPA in the eager path.
    attention_impl: str = "turbo"
    # --- additive ---
    norm: str = "rmsnorm"


@dataclass
class ModelConfig:
    model_type: str = "dlrm"
    embedding_dim: int = 64
    interaction_type: str = "concat_mlp"
    bottom_mlp_dims: list[int] = field(default_factory=lambda: [64])
    top_mlp_dims: list[int] = field(default_factory=lambda: [128, 64])
    dcn_num_cross_layers: int = 3
    dropout: float = 0.1
    embedding_init: str = "uniform"
    embedding_tables: list[EmbeddingTableConfig] = field(default_factory=list)
    cross_features: list[CrossFeatureSpec] = field(default_factory=list)
    transformer: TransformerConfig = field(default_factory=TransformerConfig)
    # --- additive ---
    # 0 = full-rank DCNv2 cross (reference); r > 0 = W ~ U V^T of rank r
    dcn_low_rank: int = 0
    # "two_tower" (reference DLRM++) or "criteo" (dense->bottom MLP, sparse ids)
    dlrm_layout: str = "two_tower"

    def resolved_embedding_tables(self) -> list[EmbeddingTableConfig]:
        """Tables with ``embedding_dim == 0`` inherit ``model.embedding_dim``."""
        return [
            dataclasses.replace(
                t, embedding_dim=t.embedding_dim if t.embedding_dim > 0 else self.embedding_dim)
            for t in self.embedding_tables
        ]


# ---------------------------------------------------------------------------
# training / distributed
# ---------------------------------------------------------------------------

@dataclass
class TrainConfig:
    batch_size: int = 256
    lr: float = 1e-3
    embedding_lr: float = 1e-2
    embedding_optimizer: str = "adam"
    embedding_eps: float = 1e-8
    weight_decay: float = 1e-5
    epochs: int = 10
    warmup_steps: int = 1000
    warmup_start_factor: float = 0.01
    sparse_warmup_steps: int = 0
    sparse_warmup_value: float = 0.1
    bf16: bool = True
    allow_tf32: bool = False
    grad_clip: float = 1.0
    shuffle: bool = True
    log_interval: int = 100
    log_max_gpu_memory: bool = False
    eval_interval: int = 1
    checkpoint_dir: str = "results"
    # declared twice in the reference; the effective default is False
    save_checkpoint: bool = False
    seed: int = 42
    loss_weights: dict[str, float] = field(default_factory=lambda: {"task0": 1.0})
    regression_tasks: list[str] = field(default_factory=list)
    dense_optimizer: str = "adamw"
    shampoo_precondition_frequency: int = 1000
    shampoo_max_preconditioner_dim: int = 4096
    shampoo_use_bf16_factor_matrix: bool = False
    shampoo_momentum: float = 0.0
    shampoo_use_nesterov: bool = False
    shampoo_use_decoupled_weight_decay: bool = False
    shampoo_use_ddp_distributed_config: bool = False
    shampoo_ddp_num_trainers_per_group: int = -1
    shampoo_ddp_communicate_params: bool = False
    torch_compile: bool = False
    torch_compile_backend: str = "inductor"
    contrastive_weight: float = 0.0
    contrastive_temperature: float = 0.1
    # --- additive ---
    # "native": sm_100a kernels on the hot path; "eager": plain PyTorch ops
    kernels: str = "native"
    eval_num_candidates: int = 5000
    # NaN/Inf guard on the loss: skip the optimizer step when non-finite
    nan_guard: bool = False
    # host watchdog: seconds a step may take before the trainer raises (0 = off)
    step_timeout_s: float = 0.0
    # peer heartbeats in the process group's store: a peer silent for this
    # many seconds (or one that reported a failure) stops the others between
    # steps with PeerFailure (0 = off)
    heartbeat_timeout_s: float = 0.0


@dataclass
class TopologyConfig:
    hbm_cap_gb: Optional[float] = None
    ddr_cap_gb: Optional[float] = None
    local_world_size: Optional[int] = None


@dataclass
class EmbeddingShardingConfig:
    enabled: bool = False
    strategy: str = "auto"
    default_table_sharding: Optional[TableShardingSpec] = None
    topology: TopologyConfig = field(default_factory=TopologyConfig)


@dataclass
class DistributedConfig:
    enabled: bool = False
    dense_strategy: str = "ddp"
    embedding_sharding: EmbeddingShardingConfig = field(default_factory=EmbeddingShardingConfig)
    num_nodes: int = 1
    gpus_per_node: int = 8
    # --- additive: "peer" = NVLink peer-memory kernels, "nccl" = baseline ---
    comm: str = "peer"


# ---------------------------------------------------------------------------
# top level
# ---------------------------------------------------------------------------

@dataclass
class Config:
    feature: FeatureConfig = field(default_factory=FeatureConfig)
    data: DataConfig = field(default_factory=DataConfig)
    model: ModelConfig = field(default_factory=ModelConfig)
    train: TrainConfig = field(default_factory=TrainConfig)
    distributed: DistributedConfig = field(default_factory=DistributedConfig)

    @property
    def task_names(self) -> list[str]:
        """Tasks with a positive loss weight (``primus_dlrm/config.py:622-626``)."""
        active = [k for k, v in self.train.loss_weights.items() if v > 0]
        return active or ["task0"]

    def feature_to_batch_key(self) -> dict[str, str]:
        """Inverse of ``schema.batch_to_feature``; identity for unmapped features."""
        inv = {feat: key for key, feat in self.schema.batch_to_feature.items()}
        for name in self.feature.all_ec_feature_names():
            inv.setdefault(name, name)
        return inv

    @property
    def schema(self) -> SchemaConfig:
        s = self.data.schema
        return s if isinstance(s, SchemaConfig) else SchemaConfig()

    def sequence_length_total(self) -> int:
        return sum(self.data.group_length(g) for g in self.feature.sequence_groups)

    def expand_cross_features(self) -> list[CrossFeatureSpec]:
        """Register each enabled cross spec as a table + scalar feature + batch
        key (+ kjt entry when an explicit order exists).  Idempotent; raises
        ``ValueError`` for collisions, unknown keys and missing fields.
        Behaviour contract: ``primus_dlrm/config.py:636-732``.
        """
        if isinstance(self.data.schema, str):
            return []
        done: set[str] = getattr(self, "_cross_registered", set())
        tables = {t.name for t in self.model.embedding_tables}
        scalars = set(self.feature.scalar_feature_names)
        expanded = []
        for spec in self.model.cross_features:
            if not spec.enabled:
                continue
            if not spec.name:
                raise ValueError("CrossFeatureSpec.name is required")
            if spec.num_embeddings <= 0:
                raise ValueError(f"CrossFeatureSpec '{spec.name}' needs num_embeddings > 0")
            if not spec.keys or len(spec.keys) < 2:
                raise ValueError(
                    f"CrossFeatureSpec '{spec.name}' needs at least 2 keys, got {spec.keys}")
            bad = [k for k in spec.keys if k not in CROSS_FEATURE_KEYS]
            if bad:
                raise ValueError(
                    f"CrossFeatureSpec '{spec.name}' uses unknown key '{bad[0]}'; "
                    f"recognized keys: {CROSS_FEATURE_KEYS}")
            if spec.name in done:
                continue
            if spec.name in tables:
                raise ValueError(
                    f"CrossFeatureSpec '{spec.name}' collides with an existing "
                    f"native embedding table; rename the cross spec or the native table")
            if spec.name in scalars:
                raise ValueError(
                    f"CrossFeatureSpec '{spec.name}' collides with an existing "
                    f"scalar feature; rename the cross spec or the scalar feature")
            self.model.embedding_tables.append(EmbeddingTableConfig(
                name=spec.name, features=[spec.name], num_embeddings=spec.num_embeddings,
                embedding_dim=0, pooling="none", sharding=spec.sharding))
            self.feature.scalar_features.append(ScalarFeatureSpec(name=spec.name))
            schema = self.data.schema
            schema.batch_to_feature.setdefault(f"{spec.name}_id", spec.name)
            if schema.kjt_feature_order and spec.name not in schema.kjt_feature_order:
                schema.kjt_feature_order.append(spec.name)
            tables.add(spec.name)
            scalars.add(spec.name)
            done.add(spec.name)
            expanded.append(spec)
        self._cross_registered = done
        return expanded

    def to_dict(self) -> dict:
        return asdict(self)

    def save(self, path: str | Path) -> None:
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        with open(path, "w") as f:
            yaml.dump(asdict(self), f, default_flow_style=False, sort_keys=False)

    @classmethod
    def from_dict(cls, raw: dict | None, base_dir: Path | None = None) -> "Config":
        if isinstance(raw, dict) and "cross_features" in (raw.get("data") or {}):
            raise ValueError(
                "'cross_features' moved from 'data.cross_features' to "
                "'model.cross_features'; please move the block under model:.")
        cfg = build_dataclass(cls, raw)
        if isinstance(cfg.data.schema, str) and cfg.data.schema:
            sp = Path(cfg.data.schema)
            if not sp.is_absolute() and base_dir is not None:
                sp = base_dir / sp
            with open(sp) as f:
                cfg.data.schema = build_dataclass(SchemaConfig, yaml.safe_load(f) or {})
        elif isinstance(cfg.data.schema, str):
            cfg.data.schema = SchemaConfig()
        cfg.expand_cross_features()
        return cfg

    @classmethod
    def load(cls, path: str | Path) -> "Config":
        path = Path(path)
        with open(path) as f:
            raw = yaml.safe_load(f)
        try:
            return cls.from_dict(raw, base_dir=path.parent)
        except ValueError as e:
            if "cross_features" in str(e) and "moved" in str(e):
                raise ValueError(f"{path}: {e}") from None
            raise


# ---------------------------------------------------------------------------
# type-hint driven loader
# ---------------------------------------------------------------------------

def _unwrap_optional(tp):
    origin = typing.get_origin(tp)
    if origin is Union:
        args = [a for a in typing.get_args(tp) if a is not type(None)]
        return args
    return [tp]


def _coerce(tp, val):
    if val is None:
        return None
    for cand in _unwrap_optional(tp):
        if dataclasses.is_dataclass(cand) and isinstance(val, dict):
            return build_dataclass(cand, val)
        origin = typing.get_origin(cand)
        if origin is list and isinstance(val, list):
            (inner,) = typing.get_args(cand) or (Any,)
            if dataclasses.is_dataclass(inner):
                return [build_dataclass(inner, v) if isinstance(v, dict) else v for v in val]
            return list(val)
        if cand is str and isinstance(val, str):
            return val
    return val


def build_dataclass(cls, raw: dict | None):
    """Instantiate dataclass ``cls`` from a nested dict, ignoring unknown keys."""
    if raw is None:
        return cls()
    hints = typing.get_type_hints(cls)
    kwargs = {}
    for f in dataclasses.fields(cls):
        if f.name in raw:
            kwargs[f.name] = _coerce(hints[f.name], raw[f.name])
    return cls(**kwargs)

"""Parameter / memory summary logged at start-up
(``primus_dlrm/utils/model_params.py``): dense parameters bucketed by model
component, embedding tables from the config (global, unsharded sizes), and
an optimizer-state memory estimate."""
from __future__ import annotations

import logging

import torch
import torch.nn as nn

logger = logging.getLogger(__name__)

_OPT_STATE_PER_PARAM = {"adamw": 2, "adam": 2, "shampoo": 4, "row_wise_adagrad": 0, "adagrad": 1, "sgd": 0}


def dtype_bytes(dt: torch.dtype) -> int:
    return torch.empty(0, dtype=dt).element_size()


def is_embedding_param(name: str) -> bool:
    """Embedding tables live under ``emb.ec.`` / ``emb.ebc.`` (learned position
    tables ``pos_emb`` are dense)."""
    return any(tok in name for tok in ("ebc.", "ec.", "embedding_bags.", ".embeddings."))


def classify_dense_param(name: str) -> str:
    n = name.lower()
    if "blocks." in n:
        return "transformer-blocks"
    if "tokenizer" in n:
        return "tokenizers"
    if "dense_proj" in n:
        return "dense-projections"
    if "head_proj" in n or n.startswith("heads.") or ".heads." in n:
        return "heads"
    if "contrastive" in n:
        return "contrastive"
    if "norm" in n:
        return "top-level norms"
    if "mlp" in n or "interaction" in n:
        return "mlps"
    return "other"


def count_embedding_params_from_config(config) -> tuple[int, int, list[tuple[str, int, int, str]]]:
    """(total params, total bytes, [(table, rows, dim, dtype)]) -- fp32 tables."""
    rows, n_tot, b_tot = [], 0, 0
    for t in config.model.resolved_embedding_tables():
        n = t.num_embeddings * t.embedding_dim
        n_tot += n
        b_tot += n * 4
        rows.append((t.name, t.num_embeddings, t.embedding_dim, "float32"))
    return n_tot, b_tot, rows


def param_summary(model: nn.Module, config, world_size: int = 1) -> dict:
    buckets: dict[str, int] = {}
    dense = 0
    for name, p in model.named_parameters():
        if not p.requires_grad or is_embedding_param(name):
            continue
        buckets[classify_dense_param(name)] = buckets.get(classify_dense_param(name), 0) + p.numel()
        dense += p.numel()
    emb_n, emb_b, tables = count_embedding_params_from_config(config)
    dopt = config.train.dense_optimizer
    sopt = config.train.embedding_optimizer
    dense_state = dense * 4 * _OPT_STATE_PER_PARAM.get(dopt, 2)
    sparse_state = sum(r * (d if sopt in ("adam", "adagrad") else 1) * (2 if sopt == "adam" else 1) * 4
                       for _, r, d, _ in tables) if sopt != "sgd" else 0
    return {"dense_params": dense, "dense_buckets": buckets, "embedding_params": emb_n,
            "embedding_bytes": emb_b, "tables": tables, "dense_optimizer_state_bytes": dense_state,
            "sparse_optimizer_state_bytes": sparse_state,
            "embedding_bytes_per_rank": emb_b / max(world_size, 1)}


def log_param_summary(model: nn.Module, config, world_size: int = 1) -> dict:
    s = param_summary(model, config, world_size)
    logger.info("Parameters: dense %.2fM, embeddings %.2fM (%.2f GB fp32, %.2f GB/rank)",
                s["dense_params"] / 1e6, s["embedding_params"] / 1e6, s["embedding_bytes"] / 1e9,
                s["embedding_bytes_per_rank"] / 1e9)
    for k, v in sorted(s["dense_buckets"].items(), key=lambda kv: -kv[1]):
        logger.info("  dense %-20s %10.2fM", k, v / 1e6)
    for name, r, d, dt in s["tables"]:
        logger.info("  table %-20s %12d x %4d %s", name, r, d, dt)
    logger.info("Optimizer state: dense %.2f GB, sparse %.2f GB", s["dense_optimizer_state_bytes"] / 1e9,
                s["sparse_optimizer_state_bytes"] / 1e9)
    return s

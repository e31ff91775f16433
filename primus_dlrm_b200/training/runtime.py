"""Runtime flags, CLI overrides and the resolved-config dump
(``primus_dlrm/training/runtime.py``).

``apply_cli_overrides`` records every field a CLI flag actually changed;
``log_resolved_config`` dumps the effective YAML with ``# OVERRIDDEN``
annotations naming the source (CLI flag or environment variable) and the
value the YAML file had.
"""
from __future__ import annotations

import logging
import os
from dataclasses import asdict

import torch
import yaml

from primus_dlrm_b200.config import Config, TrainConfig

logger = logging.getLogger(__name__)

# config path -> (environment variable, type) for values read from the env
ENV_OVERRIDES: dict[tuple[str, ...], tuple[str, type]] = {
    ("distributed", "embedding_sharding", "topology", "hbm_cap_gb"): ("PRIMUS_TORCHREC_HBM_CAP_GB", float),
    ("distributed", "embedding_sharding", "topology", "ddr_cap_gb"): ("PRIMUS_TORCHREC_DDR_CAP_GB", float),
    ("distributed", "embedding_sharding", "topology", "local_world_size"): ("PRIMUS_TORCHREC_LOCAL_WORLD_SIZE", int),
}

# CLI attribute -> config path
_CLI_FIELDS = {
    "dense_strategy": ("distributed", "dense_strategy"),
    "embedding_sharding": ("distributed", "embedding_sharding", "strategy"),
    "attention_impl": ("model", "transformer", "attention_impl"),
    "comm": ("distributed", "comm"),
    "kernels": ("train", "kernels"),
}


def configure_runtime(tc: TrainConfig) -> None:
    torch.backends.cuda.matmul.allow_tf32 = tc.allow_tf32
    torch.backends.cudnn.allow_tf32 = tc.allow_tf32
    logger.info("allow_tf32=%s", tc.allow_tf32)


def _get(cfg, path):
    node = cfg
    for k in path:
        node = getattr(node, k)
    return node


def _set(cfg, path, v):
    node = cfg
    for k in path[:-1]:
        node = getattr(node, k)
    setattr(node, path[-1], v)


def apply_cli_overrides(config: Config, args) -> Config:
    """Apply the CLI flags that map onto config fields; remember what changed."""
    changed: dict[tuple[str, ...], dict] = {}
    for attr, path in _CLI_FIELDS.items():
        val = getattr(args, attr, None)
        if val is None:
            continue
        old = _get(config, path)
        if old == val:
            continue
        changed[path] = {"yaml": old, "new": val, "src": f"--{attr.replace('_', '-')}={val}"}
        _set(config, path, val)
    if changed:
        logger.info("CLI overrides applied: %s",
                    ", ".join(f"{'.'.join(p)}={d['new']}" for p, d in changed.items()))
    config._cli_overrides = changed
    return config


def detect_env_overrides(effective: dict) -> dict[tuple[str, ...], dict]:
    found = {}
    for path, (name, typ) in ENV_OVERRIDES.items():
        raw = (os.environ.get(name) or "").strip()
        if not raw:
            continue
        try:
            val = typ(raw)
        except ValueError:
            continue
        node = effective
        for k in path[:-1]:
            node = node.get(k, {}) if isinstance(node, dict) else {}
        if not isinstance(node, dict) or node.get(path[-1]) == val:
            continue
        found[path] = {"yaml": node.get(path[-1]), "new": val, "src": f"env {name}={raw}"}
        node[path[-1]] = val
    return found


def annotate_yaml(rendered: str, overrides: dict[tuple[str, ...], dict]) -> str:
    """Append ``# OVERRIDDEN (src, yaml was X)`` to the lines of overridden keys."""
    if not overrides:
        return rendered
    lines = rendered.splitlines()
    stack: list[tuple[int, str]] = []
    out = []
    for line in lines:
        stripped = line.lstrip()
        if not stripped or stripped.startswith("#") or ":" not in stripped or stripped.startswith("- "):
            out.append(line)
            continue
        indent = len(line) - len(stripped)
        key = stripped.split(":", 1)[0].strip()
        while stack and stack[-1][0] >= indent:
            stack.pop()
        path = tuple(k for _, k in stack) + (key,)
        stack.append((indent, key))
        if path in overrides:
            d = overrides[path]
            line = f"{line}  # OVERRIDDEN ({d['src']}, yaml was {d['yaml']})"
        out.append(line)
    return "\n".join(out)


def log_resolved_config(config: Config, source_path: str | None = None) -> str:
    effective = asdict(config)
    overrides = dict(getattr(config, "_cli_overrides", {}))
    overrides.update(detect_env_overrides(effective))
    text = annotate_yaml(yaml.dump(effective, default_flow_style=False, sort_keys=False), overrides)
    logger.info("Resolved config%s:\n%s", f" (from {source_path})" if source_path else "", text)
    return text

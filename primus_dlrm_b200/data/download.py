"""Yambda download (``primus_dlrm/data/download.py``): the ``yandex/yambda``
Hugging Face dataset (50m / 500m / 5b) into ``<root>/raw/<size>/`` plus the
shared metadata.  Needs the ``datasets`` package and network access; both
are optional for everything else in this package."""
from __future__ import annotations

import logging
from pathlib import Path

logger = logging.getLogger(__name__)

_FILES = ("multi_event", "embeddings", "artist_item_mapping", "album_item_mapping")


def download_yambda(data_root: str | Path, size: str = "50m") -> Path:
    if size not in ("50m", "500m", "5b"):
        raise ValueError(f"unknown Yambda size {size!r} (50m | 500m | 5b)")
    try:
        from datasets import load_dataset
    except ImportError as e:
        raise RuntimeError("downloading Yambda needs the `datasets` package and network access") from e
    root = Path(data_root)
    raw = root / "raw" / size
    raw.mkdir(parents=True, exist_ok=True)
    meta = root / "shared_metadata"
    meta.mkdir(parents=True, exist_ok=True)
    for name in _FILES:
        shared = name != "multi_event"
        dst = (meta if shared else raw) / f"{name}.parquet"
        if dst.exists():
            continue
        data_dir = None if shared else f"flat/{size}"
        ds = load_dataset("yandex/yambda", data_dir=data_dir, data_files=f"{name}.parquet", split="train")
        ds.to_parquet(str(dst))
        logger.info("downloaded %s", dst)
    return raw

#!/usr/bin/env python3
"""Download Yambda from the Hugging Face hub (reference ``scripts/download_data.py``)."""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from primus_dlrm_b200.data.download import download_yambda  # noqa: E402


def main(argv=None):
    p = argparse.ArgumentParser(description="Download the Yambda dataset")
    p.add_argument("--data-dir", default="data/raw", help="raw-data directory (files go to <data-dir>/<size>/)")
    p.add_argument("--size", default="50m", choices=["50m", "500m", "5b"])
    a = p.parse_args(argv)
    # download_yambda takes the data root: <root>/raw/<size>, <root>/shared_metadata
    return download_yambda(Path(a.data_dir).resolve().parent, a.size)


if __name__ == "__main__":
    main()

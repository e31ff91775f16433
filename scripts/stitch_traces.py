#!/usr/bin/env python3
"""Trace analysis CLI: `stitch` report of `primus_dlrm_b200.training.trace_analysis`
(reference `scripts/stitch_traces.py`)."""
from __future__ import annotations

import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from primus_dlrm_b200.training.trace_analysis import main  # noqa: E402

if __name__ == "__main__":
    main(["stitch"] + sys.argv[1:])

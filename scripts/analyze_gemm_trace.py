#!/usr/bin/env python3
"""Trace analysis CLI: `gemm` report of `primus_dlrm_b200.training.trace_analysis`
(reference `scripts/analyze_gemm_trace.py`)."""
from __future__ import annotations

import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from primus_dlrm_b200.training.trace_analysis import main  # noqa: E402

if __name__ == "__main__":
    main(["gemm"] + sys.argv[1:])

"""Named ranges for the training step's phases.

``phase(name)`` opens an NVTX range (visible to Nsight tools) and a
``torch.profiler.record_function`` label (visible in the Chrome traces the
tracer writes), so trace tools can attribute kernels to forward, backward,
dense gradient sync and optimizer. Both cost a few microseconds per range and
nothing on the device. Set ``PD_NVTX=0`` to turn them off.
"""
from __future__ import annotations

import contextlib
import os

import torch

_ENABLED = os.environ.get("PD_NVTX", "1") != "0"


@contextlib.contextmanager
def phase(name: str):
    if not _ENABLED:
        yield
        return
    cuda = torch.cuda.is_available()
    if cuda:
        torch.cuda.nvtx.range_push(name)
    try:
        with torch.profiler.record_function(name):
            yield
    finally:
        if cuda:
            torch.cuda.nvtx.range_pop()

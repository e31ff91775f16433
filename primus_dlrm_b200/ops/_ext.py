"""Loader for the in-tree sm_100a extensions.

``core()`` returns the ``_C`` module (embedding, norm, loss, optimizer
kernels) and ``gemm()`` the ``_gemm`` module (tcgen05 GEMMs, attention).
On a machine with a CUDA device a missing or stale extension raises: a GPU
run never silently falls back to eager PyTorch.  Without a CUDA device the
eager implementations in ``primus_dlrm_b200.ops`` are the only path (they
also serve as the fp32 oracles of the kernel tests).
"""
from __future__ import annotations

import importlib
import os

import torch

_cache: dict[str, object] = {}


def _load(name: str):
    if name in _cache:
        return _cache[name]
    try:
        mod = importlib.import_module(f"primus_dlrm_b200.{name}")
    except ImportError as e:  # pragma: no cover - exercised on GPU boxes only
        src = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                           "csrc", "gemm_bindings.cpp" if name == "_gemm" else "bindings.cpp")
        if torch.cuda.is_available() and os.path.exists(src):
            raise RuntimeError(
                f"primus_dlrm_b200.{name} is not built; run `python setup.py build_ext --inplace` "
                f"(sm_100a). A CUDA device is present, so no eager fallback is used.") from e
        mod = None
    _cache[name] = mod
    return mod


def core():
    return _load("_C")


def gemm():
    return _load("_gemm")


def native_enabled(device: torch.device | str | None = None) -> bool:
    """Native kernels run for CUDA tensors unless PD_KERNELS=eager."""
    if os.environ.get("PD_KERNELS", "") == "eager":
        return False
    if device is not None and torch.device(device).type != "cuda":
        return False
    return torch.cuda.is_available()

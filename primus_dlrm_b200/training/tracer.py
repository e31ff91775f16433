"""Step-windowed torch.profiler capture (``primus_dlrm/training/tracer.py``).

For every requested step ``s`` the schedule records ``[s - warmup, s)`` as
warm-up and ``[s, s + active)`` as active, saving one Chrome trace per
window as ``trace_step{s}[_rank{r}].json``.  The step's phases carry NVTX
ranges and profiler labels (``pd.forward``, ``pd.backward``, ``pd.dense_sync``,
``pd.optimizer``; ``primus_dlrm_b200.utils.nvtx``) so trace tools can
attribute kernels to them.
"""
from __future__ import annotations

from pathlib import Path
from typing import Sequence

from torch.profiler import ProfilerAction, ProfilerActivity, profile, schedule


def window_schedule(trace_steps: Sequence[int], warmup: int, active: int):
    """Profiler schedule with one (warm-up, active) window per requested step."""
    spans = sorted((s - warmup, s, s + active) for s in trace_steps)

    def fn(step: int) -> ProfilerAction:
        for w0, a0, a1 in spans:
            if w0 <= step < a0:
                return ProfilerAction.WARMUP
            if a0 <= step < a1 - 1:
                return ProfilerAction.RECORD
            if step == a1 - 1:
                return ProfilerAction.RECORD_AND_SAVE
        return ProfilerAction.NONE

    return fn


class Tracer:
    def __init__(self, trace_dir: str | Path, trace_steps: list[int] | None = None, wait: int = 0,
                 warmup: int = 5, active: int = 10, repeat: int = 1, rank: int | None = None):
        self.trace_dir = Path(trace_dir)
        self.trace_dir.mkdir(parents=True, exist_ok=True)
        self._steps = sorted(trace_steps) if trace_steps else None
        self._rank = rank
        self._n = 0
        sched = window_schedule(self._steps, warmup, active) if self._steps else \
            schedule(wait=wait, warmup=warmup, active=active, repeat=repeat)
        self._prof = profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA], schedule=sched,
                             on_trace_ready=self._export, record_shapes=True, with_stack=False)
        self._prof.__enter__()

    def step(self) -> None:
        self._prof.step()

    def stop(self) -> None:
        self._prof.__exit__(None, None, None)

    def _export(self, prof) -> None:
        suffix = f"_rank{self._rank}" if self._rank is not None else ""
        if self._steps and self._n < len(self._steps):
            path = self.trace_dir / f"trace_step{self._steps[self._n]}{suffix}.json"
        else:
            path = self.trace_dir / f"trace_{self._n}{suffix}.json"
        prof.export_chrome_trace(str(path))
        self._n += 1

    @property
    def trace_files(self) -> list[Path]:
        return sorted(self.trace_dir.glob("trace_*.json"))


def parse_trace_ranks(spec: str | None) -> set[int] | None:
    """``""``/``None`` -> {0}; ``"all"`` -> None (every rank); ``"0,3"`` -> {0, 3}."""
    if not spec:
        return {0}
    s = spec.strip().lower()
    if s == "all":
        return None
    out = {int(t) for t in s.split(",") if t.strip()}
    return out or {0}

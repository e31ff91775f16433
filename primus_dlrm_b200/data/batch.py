"""Packed host->device batches.

A training batch is a dict of many small tensors (13 id features, dense
features, labels).  ``PackedBatch`` lays them out in ONE pinned host buffer
(256-byte aligned slots, ids narrowed to int32 when they fit) so moving a
batch to the GPU is a single ``cudaMemcpyAsync`` on a copy stream, after
which the device batch is a set of views of one device buffer.

This replaces the reference's per-tensor ``.to(device, non_blocking=True)``
+ ``record_stream`` of ``PipelineBatch`` (``primus_dlrm/data/pipeline_batch.py:29-67``).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

_ALIGN = 256


@dataclass
class _Field:
    name: str
    dtype: torch.dtype
    shape: tuple[int, ...]
    offset: int
    nbytes: int


def _wire_dtype(t: torch.Tensor, narrow_ids: bool) -> torch.dtype:
    if t.dtype == torch.int64 and narrow_ids:
        if t.numel() == 0 or (int(t.max()) < 2 ** 31 and int(t.min()) >= -2 ** 31):
            return torch.int32
    if t.dtype == torch.float64:
        return torch.float32
    return t.dtype


class PackedBatch:
    """One pinned buffer holding every tensor of a batch."""

    def __init__(self, batch: dict[str, torch.Tensor], pin: bool = True, narrow_ids: bool = True):
        fields, off = [], 0
        for k, v in batch.items():
            if not isinstance(v, torch.Tensor):
                continue
            dt = _wire_dtype(v, narrow_ids)
            nb = v.numel() * torch.empty(0, dtype=dt).element_size()
            fields.append(_Field(k, dt, tuple(v.shape), off, nb))
            off += (nb + _ALIGN - 1) // _ALIGN * _ALIGN
        self.fields = fields
        self.nbytes = max(off, _ALIGN)
        buf = torch.empty(self.nbytes, dtype=torch.uint8)
        self.host = buf.pin_memory() if (pin and torch.cuda.is_available()) else buf
        for f in fields:
            self._view(self.host, f).copy_(batch[f.name].to(f.dtype))

    @staticmethod
    def _view(buf: torch.Tensor, f: _Field) -> torch.Tensor:
        return buf[f.offset:f.offset + f.nbytes].view(f.dtype).view(f.shape)

    def views(self, buf: torch.Tensor) -> dict[str, torch.Tensor]:
        return {f.name: self._view(buf, f) for f in self.fields}

    def to_device(self, device, out: torch.Tensor | None = None,
                  stream: torch.cuda.Stream | None = None) -> dict[str, torch.Tensor]:
        """Copy to ``device`` (into ``out`` if given) with one async copy."""
        if out is None:
            out = torch.empty(self.nbytes, dtype=torch.uint8, device=device)
        if stream is not None:
            with torch.cuda.stream(stream):
                out.copy_(self.host, non_blocking=True)
        else:
            out.copy_(self.host, non_blocking=True)
        return self.views(out)

    def host_views(self) -> dict[str, torch.Tensor]:
        return self.views(self.host)


class DeviceBatchStager:
    """Double-buffered H2D staging on a side stream.

    ``stage(packed)`` starts the copy of the next batch; ``get()`` makes the
    compute stream wait for it and returns the device views.  The buffer of a
    batch is reused two batches later, after the compute stream has passed
    an event recorded behind it.
    """

    def __init__(self, device, nbytes: int):
        self.device = torch.device(device)
        self.stream = torch.cuda.Stream(device=self.device)
        self.bufs = [torch.empty(nbytes, dtype=torch.uint8, device=self.device) for _ in range(2)]
        self.free = [torch.cuda.Event() for _ in range(2)]
        self.ready = [torch.cuda.Event() for _ in range(2)]
        self.i = 0
        self.pending = None
        self.in_use = None  # buffer index handed to the compute stream last

    def stage(self, packed: PackedBatch) -> None:
        k = self.i % 2
        self.i += 1
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(self.free[k])
            self.bufs[k][:packed.nbytes].copy_(packed.host, non_blocking=True)
            self.ready[k].record(self.stream)
        self.pending = (k, packed)

    def get(self) -> dict[str, torch.Tensor]:
        k, packed = self.pending
        cur = torch.cuda.current_stream(self.device)
        if self.in_use is not None:
            # everything that reads the previous buffer is already enqueued
            self.free[self.in_use].record(cur)
        cur.wait_event(self.ready[k])
        self.in_use = k
        return packed.views(self.bufs[k])

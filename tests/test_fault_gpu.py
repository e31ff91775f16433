"""Bounded device waits on one GPU: the peer barrier's spin on a flag that
nothing sets gives up at its time limit, records ``kWaitTimeout`` (2) in the
error word and returns, and the context stays usable.  The flag pads are two
local buffers, so no other rank or kernel is involved."""
from __future__ import annotations

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("timeout_ns", [0, int(0.2e9)])
def test_barrier_wait_runs_out_and_reports(timeout_ns):
    from primus_dlrm_b200.ops import _ext
    dev = torch.device("cuda", 0)
    pads = [torch.zeros(64, dtype=torch.int64, device=dev) for _ in range(2)]
    ptrs = torch.tensor([p.data_ptr() for p in pads], dtype=torch.int64)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    t0 = time.monotonic()
    _ext.core().signal_barrier(ptrs, 0, 7, timeout_ns, err)   # "rank 1" never arrives
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    assert int(err.item()) == 2
    assert waited < 5.0
    # our own arrival was published into both pads before the wait
    assert int(pads[0][0].item()) == 7 and int(pads[1][0].item()) == 7
    # the context is intact
    x = torch.randn(256, 256, device=dev)
    torch.testing.assert_close((x @ torch.eye(256, device=dev)).cpu(), x.cpu())


def test_barrier_completes_when_flags_are_set():
    from primus_dlrm_b200.ops import _ext
    dev = torch.device("cuda", 0)
    pads = [torch.zeros(64, dtype=torch.int64, device=dev) for _ in range(2)]
    pads[0][1] = 9                      # "rank 1" already arrived at epoch 9
    ptrs = torch.tensor([p.data_ptr() for p in pads], dtype=torch.int64)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    _ext.core().signal_barrier(ptrs, 0, 9, int(1e9), err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0

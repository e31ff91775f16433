"""Resume restores this process's CUDA generator (dropout and on-device
sampling draw from it), so a resumed run continues the same random stream."""
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

CONFIGS = Path(__file__).resolve().parent.parent / "configs"


def test_resume_restores_cuda_rng_state(tmp_path):
    from primus_dlrm_b200.config import Config
    from primus_dlrm_b200.models.onetrans import OneTransModel
    from primus_dlrm_b200.training.checkpoint import load_checkpoint, save_checkpoint

    cfg = Config.load(CONFIGS / "onetrans_tiny.yaml")
    model = OneTransModel(cfg)
    torch.cuda.manual_seed(123)
    torch.rand(7, device="cuda")                      # advance the stream
    path = save_checkpoint(tmp_path / "epoch_0.pt", model, epoch=0, global_step=3)
    expect = torch.rand(1000, device="cuda")
    torch.rand(5000, device="cuda")                   # move it elsewhere
    load_checkpoint(path, model)
    got = torch.rand(1000, device="cuda")
    assert torch.equal(got, expect)

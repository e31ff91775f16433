"""Training stack on CPU: engine steps, checkpoint save / resume (bit-exact
continuation), corrupted-checkpoint errors, the training and eval CLIs,
config override annotation, the profiler window tracer, the host watchdog,
parameter accounting and ranking evaluation.

Reference behaviour: ``primus_dlrm/training/dist_trainer.py`` (loop, logs,
checkpoint layout), ``primus_dlrm/training/tracer.py``,
``primus_dlrm/training/runtime.py``, ``scripts/run_distributed.py``,
``scripts/eval_checkpoint.py``.
"""
from __future__ import annotations

import importlib.util
import sys
import time
from argparse import Namespace
from pathlib import Path

import pytest
import torch

from primus_dlrm_b200.config import Config

ROOT = Path(__file__).resolve().parent.parent
CONFIGS = ROOT / "configs"


def _tiny(steps_cfg=None) -> Config:
    c = Config.load(CONFIGS / "onetrans_tiny.yaml")
    c.data.history_length = 8
    c.train.batch_size = 32
    c.train.kernels = "eager"
    return c


def _engine(cfg, seed=0):
    from primus_dlrm_b200.models.onetrans import OneTransModel
    from primus_dlrm_b200.training.engine import TrainEngine
    torch.manual_seed(seed)
    model = OneTransModel(cfg)
    return model, TrainEngine(model, cfg, torch.device("cpu"), total_steps=100)


def _batches(cfg, n):
    from primus_dlrm_b200.data.synthetic import generate_batch
    return [generate_batch(cfg, 32, seed=100 + i) for i in range(n)]


def _load_script(name):
    spec = importlib.util.spec_from_file_location(f"_script_{name}", ROOT / "scripts" / f"{name}.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_engine_reduces_loss():
    cfg = _tiny()
    cfg.train.warmup_steps = 1
    cfg.train.lr = 3e-3
    model, eng = _engine(cfg)
    b = _batches(cfg, 1)[0]
    first = float(eng.step(b)[0])
    for _ in range(15):
        last = float(eng.step(b)[0])
    assert last < first
    assert eng.global_step == 16


def test_nan_guard_skips_step():
    cfg = _tiny()
    cfg.train.nan_guard = True
    model, eng = _engine(cfg)
    b = _batches(cfg, 1)[0]
    b["audio_embed"] = torch.full_like(b["audio_embed"], float("nan"))
    before = [p.detach().clone() for p in model.heads.parameters()]
    eng.step(b)
    assert eng.skipped_steps == 1
    for p, q in zip(model.heads.parameters(), before):
        assert torch.equal(p.detach(), q)


@pytest.mark.parametrize("sparse_opt", ["row_wise_adagrad", "adam"])
def test_checkpoint_resume_is_bit_exact(tmp_path, sparse_opt):
    from primus_dlrm_b200.training.checkpoint import load_checkpoint, save_checkpoint
    cfg = _tiny()
    cfg.train.embedding_optimizer = sparse_opt
    data = _batches(cfg, 6)
    model, eng = _engine(cfg)
    for b in data[:3]:
        eng.step(b)
    ck = save_checkpoint(tmp_path / "checkpoints" / "epoch_0.pt", model, 0, eng.global_step, engine=eng, config=cfg)
    ref = [float(eng.step(b)[0]) for b in data[3:]]

    model2, eng2 = _engine(cfg, seed=123)            # different init: everything must come from the file
    ckpt = load_checkpoint(ck, model2, eng2)
    assert ckpt["global_step"] == 3 and eng2.global_step == 3
    got = [float(eng2.step(b)[0]) for b in data[3:]]
    assert got == ref
    # the reference's keys are present
    assert {"epoch", "global_step", "model_state_dict"} <= set(ckpt)


def test_checkpoint_corrupt_and_foreign_files(tmp_path):
    from primus_dlrm_b200.training.checkpoint import latest_checkpoint, load_checkpoint, save_checkpoint
    cfg = _tiny()
    model, eng = _engine(cfg)
    d = tmp_path / "run"
    for e in (0, 2, 10):
        save_checkpoint(d / "checkpoints" / f"epoch_{e}.pt", model, e, e, engine=eng)
    assert latest_checkpoint(d).name == "epoch_10.pt"
    assert not list((d / "checkpoints").glob(".*tmp*"))   # atomic writes leave no temporaries
    bad = tmp_path / "bad.pt"
    raw = (d / "checkpoints" / "epoch_0.pt").read_bytes()
    bad.write_bytes(raw[: len(raw) // 3])
    with pytest.raises(RuntimeError, match="bad.pt"):
        load_checkpoint(bad, model)
    torch.save({"weights": 1}, tmp_path / "foreign.pt")
    with pytest.raises(RuntimeError, match="not a training checkpoint"):
        load_checkpoint(tmp_path / "foreign.pt", model)
    # weights-only checkpoints (the reference's layout) load without resume state
    torch.save({"epoch": 0, "global_step": 7, "model_state_dict": model.state_dict()}, tmp_path / "w.pt")
    m2, e2 = _engine(cfg, seed=5)
    load_checkpoint(tmp_path / "w.pt", m2, e2)
    assert e2.global_step == 7
    for (n1, p1), (n2, p2) in zip(model.state_dict().items(), m2.state_dict().items()):
        assert n1 == n2 and torch.equal(p1, p2)


def test_training_cli_checkpoint_resume_and_eval(tmp_path, monkeypatch):
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT"):
        monkeypatch.delenv(k, raising=False)
    cfg = _tiny()
    cfg.train.save_checkpoint = True
    cfg.train.epochs = 2
    cfg.data.synthetic.num_prebatched = 2
    p = tmp_path / "cfg.yaml"
    cfg.save(p)
    rd = _load_script("run_distributed")
    res = tmp_path / "results"
    rd.main(["--config", str(p), "--max-steps", "4", "--log-interval", "2", "--results-dir", str(res),
             "--run-name", "r", "--skip-eval", "--kernels", "eager"])
    cks = sorted((res / "r" / "checkpoints").glob("epoch_*.pt"))
    assert [c.name for c in cks] == ["epoch_0.pt"]
    assert "global_throughput" in (res / "r" / "logs" / "train.log").read_text()
    ck = torch.load(cks[0], weights_only=False)
    assert ck["global_step"] == 4
    # resume continues the step count from the file
    rd.main(["--config", str(p), "--max-steps", "6", "--log-interval", "1", "--results-dir", str(res),
             "--run-name", "r", "--skip-eval", "--kernels", "eager", "--resume", "latest"])
    ck = torch.load(res / "r" / "checkpoints" / "epoch_0.pt", weights_only=False)
    assert ck["global_step"] == 6
    # the eval CLI scores the checkpoint on synthetic users
    ev = _load_script("eval_checkpoint")
    rg, rp = ev.main(["--config", str(p), "--checkpoint", str(res / "r" / "checkpoints" / "epoch_0.pt"),
                      "--synthetic-users", "4", "--num-candidates", "64"])
    assert 0.0 <= rg["ndcg@10"] <= 1.0 and 0.0 <= rp["recall@100"] <= 1.0


def test_cli_overrides_are_annotated():
    from primus_dlrm_b200.training.runtime import apply_cli_overrides, log_resolved_config
    cfg = Config.load(CONFIGS / "onetrans_tiny.yaml")
    args = Namespace(dense_strategy="fsdp", embedding_sharding=None, attention_impl="sdpa", comm="nccl",
                     kernels=None)
    apply_cli_overrides(cfg, args)
    assert cfg.distributed.dense_strategy == "fsdp" and cfg.distributed.comm == "nccl"
    text = log_resolved_config(cfg)
    line = [l for l in text.splitlines() if l.strip().startswith("dense_strategy:")][0]
    assert "OVERRIDDEN (--dense-strategy=fsdp, yaml was ddp)" in line
    # unchanged values (attention_impl already sdpa) are not annotated
    assert "--attention-impl" not in text


def test_env_override_annotation(monkeypatch):
    from primus_dlrm_b200.training.runtime import log_resolved_config
    monkeypatch.setenv("PRIMUS_TORCHREC_HBM_CAP_GB", "80")
    text = log_resolved_config(Config.load(CONFIGS / "onetrans_tiny.yaml"))
    assert any("hbm_cap_gb" in l and "OVERRIDDEN (env PRIMUS_TORCHREC_HBM_CAP_GB=80" in l for l in text.splitlines())


def test_parse_trace_ranks_and_window_schedule():
    from torch.profiler import ProfilerAction

    from primus_dlrm_b200.training.tracer import parse_trace_ranks, window_schedule
    assert parse_trace_ranks("") == {0}
    assert parse_trace_ranks("all") is None
    assert parse_trace_ranks("0, 3") == {0, 3}
    f = window_schedule([10], warmup=2, active=3)
    acts = [f(s) for s in range(7, 15)]
    assert acts == [ProfilerAction.NONE, ProfilerAction.WARMUP, ProfilerAction.WARMUP, ProfilerAction.RECORD,
                    ProfilerAction.RECORD, ProfilerAction.RECORD_AND_SAVE, ProfilerAction.NONE, ProfilerAction.NONE]


def test_tracer_writes_a_trace(tmp_path):
    from primus_dlrm_b200.training.tracer import Tracer
    t = Tracer(tmp_path / "trace", trace_steps=[2], warmup=1, active=2, rank=0)
    x = torch.randn(64, 64)
    for _ in range(6):
        x = x @ x.t() / 64
        t.step()
    t.stop()
    assert [p.name for p in t.trace_files] == ["trace_step2_rank0.json"]


def test_watchdog_fires_and_kicks():
    from primus_dlrm_b200.training.trainer import Watchdog
    fired = []
    w = Watchdog(0.4, on_timeout=lambda: fired.append(time.monotonic()))
    time.sleep(0.8)              # not armed before the first kick
    assert not fired
    for _ in range(4):           # kicked: never fires
        time.sleep(0.15)
        w.kick()
    assert not fired
    time.sleep(1.2)              # not kicked: fires once
    assert len(fired) == 1 and w.fired
    w.stop()
    off = Watchdog(0.0, on_timeout=lambda: fired.append(0))
    time.sleep(0.1)
    assert len(fired) == 1
    off.stop()


def test_param_summary():
    from primus_dlrm_b200.models.onetrans import OneTransModel
    from primus_dlrm_b200.utils.model_params import classify_dense_param, is_embedding_param, param_summary
    cfg = _tiny()
    m = OneTransModel(cfg)
    s = param_summary(m, cfg, world_size=2)
    emb = sum(t.num_embeddings * t.embedding_dim for t in cfg.model.resolved_embedding_tables())
    assert s["embedding_params"] == emb
    dense = sum(p.numel() for n, p in m.named_parameters() if not is_embedding_param(n))
    assert s["dense_params"] == dense
    assert classify_dense_param("blocks.0.attn.qkv.weight") == "transformer-blocks"


def test_ranking_eval_synthetic():
    from primus_dlrm_b200.data.dataset import SyntheticEvalDataset
    from primus_dlrm_b200.evaluation.metrics import evaluate_ranking, evaluate_ranking_peruser
    from primus_dlrm_b200.models.onetrans import OneTransModel
    cfg = _tiny()
    m = OneTransModel(cfg).eval()
    ds = SyntheticEvalDataset(cfg, num_users=3, num_items_with_history=50)
    with torch.no_grad():
        g = evaluate_ranking(m, ds, torch.device("cpu"), candidate_item_ids=torch.arange(40).numpy(), ks=[5, 10])
        p = evaluate_ranking_peruser(m, ds, torch.device("cpu"), ks=[5, 10], top_n=20)
    for d in (g, p):
        assert all(0.0 <= v <= 1.0 for k, v in d.items() if isinstance(v, float))
        assert "ndcg@10" in d

"""CLI scripts and offline tools on CPU: preprocessing / cache building / full
and MostPop evaluation on a fabricated Yambda dataset, the single-device
trainer, the torchrun launcher (2 gloo ranks), and the trace analyses on a
synthetic Chrome trace with known intervals."""
from __future__ import annotations

import importlib.util
import json
import math
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
CONFIGS = ROOT / "configs"


def _script(name):
    spec = importlib.util.spec_from_file_location(f"_s_{name}", ROOT / "scripts" / f"{name}.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


# --------------------------------------------------------------------------- trace analysis

def _trace():
    # device 0: compute kernels [0,100) and [150,200); an all-reduce [80,180) of 1 MB over 4 ranks
    ev = [
        {"ph": "X", "cat": "kernel", "name": "void pd::tc::gemm_kernel<256, 3>", "pid": 0, "tid": 7, "ts": 0,
         "dur": 100, "args": {"External id": 11, "device": 0}},
        {"ph": "X", "cat": "kernel", "name": "void pd::norm_fwd_kernel<0, 1>", "pid": 0, "tid": 7, "ts": 150,
         "dur": 50, "args": {"External id": 12, "device": 0}},
        {"ph": "X", "cat": "kernel", "name": "ncclDevKernel_AllReduce_Sum_f32_RING_LL", "pid": 0, "tid": 9,
         "ts": 80, "dur": 100, "args": {"External id": 13, "device": 0}},
        {"ph": "X", "cat": "cpu_op", "name": "aten::mm", "pid": 1, "tid": 1, "ts": 0, "dur": 5,
         "args": {"External id": 11, "Input Dims": [[1024, 512], [512, 256]]}},
        {"ph": "X", "cat": "cpu_op", "name": "record_param_comms", "pid": 1, "tid": 1, "ts": 70, "dur": 5,
         "args": {"External id": 13, "In msg nelems": 262144, "Out msg nelems": 262144, "dtype": "Float",
                  "Group size": 4}},
    ]
    return {"traceEvents": ev}


def test_trace_breakdown_comms_gemm(tmp_path):
    from primus_dlrm_b200.training.trace_analysis import comm_report, gemm_report, kernel_breakdown
    tr = _trace()
    bd = kernel_breakdown(tr)
    assert bd["gemm"]["ms_per_step"] == pytest.approx(0.1)
    assert bd["norm"]["ms_per_step"] == pytest.approx(0.05)
    assert bd["communication"]["ms_per_step"] == pytest.approx(0.1)
    cr = comm_report(tr)
    ar = cr["collectives"]["all_reduce"]
    # covered by compute: [80,100) and [150,180) -> 50 us of 100 exposed
    assert ar["exposed_ms"] == pytest.approx(0.05) and cr["overlapped_ms"] == pytest.approx(0.05)
    assert ar["algbw_gbs"] == pytest.approx(1048576 / 100e-6 / 1e9, rel=1e-2)
    assert ar["busbw_gbs"] == pytest.approx(ar["algbw_gbs"] * 1.5, rel=1e-2)
    g = gemm_report(tr)
    assert g[0]["M"] == 1024 and g[0]["N"] == 256 and g[0]["K"] == 512
    assert g[0]["tflops"] == pytest.approx(2 * 1024 * 256 * 512 / 100e-6 / 1e12, rel=1e-2)


def test_idle_gaps():
    from primus_dlrm_b200.training.trace_analysis import idle_gaps
    tr = _trace()
    # device 0 busy [0, 200) through the all-reduce; add a kernel at [300, 310) after a host sync
    tr["traceEvents"].append({"ph": "X", "cat": "kernel", "name": "k", "pid": 0, "tid": 7, "ts": 300, "dur": 10,
                              "args": {"device": 0}})
    tr["traceEvents"].append({"ph": "X", "cat": "cpu_op", "name": "aten::item", "pid": 1, "tid": 1, "ts": 190,
                              "dur": 100, "args": {}})
    g = idle_gaps(tr, min_us=20)["0"]
    assert g["n_gaps"] == 1 and g["idle_ms"] == pytest.approx(0.1)
    assert g["top"][0]["host_op"] == "aten::item" and g["top"][0]["start_us"] == pytest.approx(200)
    assert g["span_ms"] == pytest.approx(0.31)


def test_stitch_traces(tmp_path):
    from primus_dlrm_b200.training.trace_analysis import stitch
    paths = []
    for r in range(2):
        p = tmp_path / f"trace_step5_rank{r}.json"
        p.write_text(json.dumps(_trace()))
        paths.append(p)
    out = stitch(paths, tmp_path / "merged.json")
    ev = json.loads(out.read_text())["traceEvents"]
    pids = {e["pid"] for e in ev}
    assert {0, 1, 1_000_000, 1_000_001} <= pids
    assert any(e.get("ph") == "M" and e["args"]["name"].startswith("rank 1") for e in ev)
    rc = subprocess.run([sys.executable, str(ROOT / "scripts" / "analyze_comms.py"), str(paths[0])],
                        capture_output=True, text=True, timeout=120)
    assert rc.returncode == 0 and "all_reduce" in rc.stdout


# --------------------------------------------------------------------------- MostPop

def test_mostpop_paper_protocol():
    from primus_dlrm_b200.evaluation.mostpop import LAST_TIMESTAMP, mostpop_paper
    t_test = LAST_TIMESTAMP - 86_400
    # train: item 5 x3, item 7 x2, item 9 x1 (listen+); user 1 and 2 in train
    uid = [1, 1, 2, 2, 2, 1, 1, 2, 3]
    item = [5, 5, 5, 7, 7, 9, 5, 9, 5]
    ts = [0, 10, 20, 30, 40, 50, t_test + 5, t_test + 9, t_test + 1]
    et = ["listen"] * 9
    pr = [90] * 9
    res = mostpop_paper(uid, item, ts, et, pr, "listen_plus", num_ranked=3, ks=(1, 3))
    # ranking [5, 7, 9]; user 1 gt {5}: ndcg@1 = 1; user 2 gt {9}: rank 3 -> 1/log2(4); user 3 not in train
    assert res["num_users"] == 2
    assert res["recall@1"] == pytest.approx(0.5)
    assert res["ndcg@3"] == pytest.approx((1.0 + 1.0 / math.log2(4)) / 2)


# --------------------------------------------------------------------------- data CLIs + eval

@pytest.fixture(scope="module")
def yroot(tmp_path_factory):
    import pyarrow as pa
    import pyarrow.parquet as pq
    root = tmp_path_factory.mktemp("ydata")
    rng = np.random.default_rng(3)
    n = 2500
    uid = rng.integers(1, 10, n)
    item = rng.integers(1, 50, n)
    ts = np.sort(rng.integers(0, 12 * 86400, n))
    et = rng.choice(["listen", "listen", "listen", "like", "dislike"], n)
    played = np.where(et == "listen", rng.integers(0, 101, n), np.nan).astype(np.float32)
    raw = root / "raw" / "50m"
    raw.mkdir(parents=True)
    pq.write_table(pa.table({"uid": uid, "item_id": item, "timestamp": ts, "event_type": et.tolist(),
                             "is_organic": np.zeros(n, np.int8), "played_ratio_pct": played,
                             "track_length_seconds": np.full(n, 180, np.int32)}), raw / "multi_event.parquet")
    items = np.arange(50)
    pq.write_table(pa.table({"item_id": items, "artist_id": items % 5}), root / "raw" / "artist_item_mapping.parquet")
    pq.write_table(pa.table({"item_id": items, "album_id": items % 9}), root / "raw" / "album_item_mapping.parquet")
    _script("preprocess").main(["--raw-dir", str(root / "raw"), "--size", "50m", "--train-days", "10"])
    return root


def _cfg(tmp_path) -> Path:
    from primus_dlrm_b200.config import Config
    c = Config.load(CONFIGS / "onetrans_tiny.yaml")
    c.data.synthetic.enabled = False
    c.data.history_length = 6
    c.data.data_dir = "unused"
    c.feature.dense_features = [d for d in c.feature.dense_features if d.name != "audio_embed"]
    for t in c.model.embedding_tables:
        t.num_embeddings = 60
    p = tmp_path / "cfg.yaml"
    c.save(p)
    return p


def test_preprocess_build_cache_and_eval(yroot, tmp_path):
    assert (yroot / "processed" / "train_sessions.parquet").exists()
    cfg = _cfg(tmp_path)
    built = _script("build_cache").main(["--config", str(cfg), "--data-root", str(yroot)])
    assert any(b.startswith("train:") for b in built) and any(b.startswith("eval:") for b in built)
    assert any((yroot / "cache").iterdir())
    ef = _script("eval_full")
    mp = ef.main(["--config", str(cfg), "--processed-dir", str(yroot / "processed"), "--mode", "mostpop"])
    assert mp["num_users"] > 0 and 0.0 <= mp["ndcg@10"] <= 1.0
    g = ef.main(["--config", str(cfg), "--processed-dir", str(yroot / "processed"), "--mode", "global",
                 "--device", "cpu", "--eval-top-k", "20"])
    assert 0.0 <= g["recall@100"] <= 1.0
    pu = ef.main(["--config", str(cfg), "--processed-dir", str(yroot / "processed"), "--mode", "peruser",
                  "--device", "cpu"])
    assert pu["num_users"] > 0
    em = _script("eval_mostpop").main(["--data-file", str(yroot / "raw" / "50m" / "multi_event.parquet")])
    assert "ndcg@10" in em


def test_single_device_train_script(tmp_path, monkeypatch):
    from primus_dlrm_b200.config import Config
    c = Config.load(CONFIGS / "onetrans_tiny.yaml")
    c.train.batch_size = 16
    c.data.history_length = 4
    c.train.kernels = "eager"
    p = tmp_path / "c.yaml"
    c.save(p)
    monkeypatch.chdir(tmp_path)
    _script("train").main(["--config", str(p), "--device", "cpu", "--max-steps", "3", "--results-dir",
                           str(tmp_path / "res"), "--skip-eval", "--log-interval", "1"])
    assert "global_throughput" in (tmp_path / "res" / "train" / "logs" / "train.log").read_text()


def test_launcher_two_gloo_ranks(tmp_path):
    from primus_dlrm_b200.config import Config
    c = Config.load(CONFIGS / "onetrans_tiny.yaml")
    c.train.batch_size = 16
    c.data.history_length = 4
    c.train.kernels = "eager"
    p = tmp_path / "c.yaml"
    c.save(p)
    from tests.dist_utils import free_port
    env = dict(os.environ, OMP_NUM_THREADS="2")
    rc = subprocess.run(["bash", str(ROOT / "scripts" / "launch_torchrun.sh"), "--config", str(p), "--gpus", "2",
                         "--master-port", str(free_port()), "--timeout", "240", "--", "--max-steps", "2",
                         "--skip-eval", "--results-dir", str(tmp_path / "r"), "--dense-strategy", "dmp",
                         "--kernels", "eager", "--log-interval", "1"],
                        capture_output=True, text=True, timeout=300, env=env, cwd=str(tmp_path))
    assert rc.returncode == 0, rc.stdout[-3000:] + rc.stderr[-3000:]
    assert "Training complete" in rc.stdout + rc.stderr

"""Data pipeline on CPU: synthetic generator, packed batches, sliding-window
counters (vs a brute-force oracle), the flat event store cache, Yambda
preprocessing -> train / eval datasets on a fabricated raw dataset, cross-id
collation and the large-dataset sampler.

Reference coverage: ``tests/test_cross_features.py`` (cache contract, collate),
``primus_dlrm/data/{synthetic,counters,dataset,preprocessing}.py`` behaviour.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from primus_dlrm_b200.config import Config, CrossFeatureSpec

CONFIGS = Path(__file__).resolve().parent.parent / "configs"


# --------------------------------------------------------------------------- synthetic

def test_generate_batch_contract():
    from primus_dlrm_b200.data.synthetic import generate_batch, table_size_by_feature
    cfg = Config.load(CONFIGS / "onetrans_tiny.yaml")
    b = generate_batch(cfg, 256, seed=3)
    f2k = cfg.feature_to_batch_key()
    sizes = table_size_by_feature(cfg)
    for f in cfg.feature.scalar_feature_names:
        t = b[f2k.get(f, f)]
        assert t.shape == (256,) and t.dtype == torch.int64
        assert int(t.min()) >= 0 and int(t.max()) < sizes[f]
    for g, feats in cfg.feature.sequence_groups.items():
        for f in feats:
            assert b[f2k.get(f, f)].shape == (256, cfg.data.group_length(g))
    for d in cfg.feature.dense_features:
        assert b[d.name].shape == (256, d.dim) and b[d.name].dtype == torch.float32
    for task in cfg.task_names:
        assert b[task].shape == (256,)
    # binary tasks are {0,1}; the regression target lies in [0, 1]
    assert set(b["listen_plus"].unique().tolist()) <= {0.0, 1.0}
    assert 0.0 <= float(b["played_ratio"].min()) and float(b["played_ratio"].max()) <= 1.0
    # deterministic in the seed
    b2 = generate_batch(cfg, 256, seed=3)
    assert all(torch.equal(b[k], b2[k]) for k in b)
    assert not torch.equal(generate_batch(cfg, 256, seed=4)["item_id"], b["item_id"])


def test_zipf_ids_are_skewed_and_in_range():
    from primus_dlrm_b200.data.synthetic import zipf_ids
    g = torch.Generator().manual_seed(0)
    ids = zipf_ids(1_000_000, (200_000,), 1.05, g)
    assert int(ids.min()) >= 0 and int(ids.max()) < 1_000_000
    _, counts = torch.unique(ids, return_counts=True)
    top = torch.sort(counts, descending=True).values
    # the hottest id carries a few percent of the mass; most ids are cold
    assert top[0].item() / ids.numel() > 0.01
    assert (counts == 1).sum().item() > 0.3 * counts.numel()


def test_synthetic_pipe_and_dataset():
    from primus_dlrm_b200.data.synthetic import SyntheticDataPipe, SyntheticDataset, collate_synthetic
    cfg = Config.load(CONFIGS / "onetrans_tiny.yaml")
    pipe = SyntheticDataPipe(cfg, 32, num_prebatched=2, seed=1)
    a, b, c = next(pipe), next(pipe), next(pipe)
    assert a is c and a is not b
    ds = SyntheticDataset(cfg)
    batch = collate_synthetic([ds[i] for i in range(4)])
    assert batch["item_id"].shape == (4,)


def test_packed_batch_roundtrip():
    from primus_dlrm_b200.data.batch import PackedBatch
    cfg = Config.load(CONFIGS / "onetrans_tiny.yaml")
    from primus_dlrm_b200.data.synthetic import generate_batch
    b = generate_batch(cfg, 64, seed=0)
    p = PackedBatch(b)
    for f in p.fields:
        assert f.offset % 256 == 0
    dev = p.to_device("cpu")
    for k, v in b.items():
        w = dev[k]
        assert w.shape == v.shape
        if v.dtype == torch.int64:
            assert w.dtype == torch.int32          # ids travel narrowed
        assert torch.equal(w.to(v.dtype), v)
    # ids that do not fit int32 keep int64
    q = PackedBatch({"x": torch.tensor([1 << 40, 3])})
    assert q.host_views()["x"].dtype == torch.int64


# --------------------------------------------------------------------------- counters

def _brute_counts(keys, ts, flags, windows_days):
    """Per event i: events j < i (in time order within the same key) whose
    ts >= ts_i - w count, for each window and each flag."""
    n = keys.size
    order = np.lexsort((ts, keys))
    rank = np.empty(n, np.int64)
    rank[order] = np.arange(n)
    out = np.zeros((n, 3 * len(windows_days)), np.float32)
    for i in range(n):
        for w, days in enumerate(windows_days):
            edge = ts[i] - days * 86400
            m = (keys == keys[i]) & (rank < rank[i]) & (ts >= edge)
            for c, f in enumerate(flags):
                out[i, 3 * w + c] = np.log1p(f[m].sum())
    return out


def test_counters_match_bruteforce():
    from primus_dlrm_b200.data import counters as C
    rng = np.random.default_rng(0)
    n = 300
    uid = rng.integers(0, 6, n)
    item = rng.integers(0, 15, n)
    ts = rng.integers(0, 40 * 86400, n)
    ts[:20] = ts[0]                                  # ties
    lp = rng.random(n) < 0.4
    like = rng.random(n) < 0.1
    skip = ~lp & (rng.random(n) < 0.5)
    win = [1, 7, 30]
    np.testing.assert_allclose(C.precompute_user_counters(uid, ts, lp, like, skip, win),
                               _brute_counts(uid, ts, (lp, like, skip), win), rtol=1e-6)
    np.testing.assert_allclose(C.precompute_item_counters(item, ts, lp, like, skip, win),
                               _brute_counts(item, ts, (lp, like, skip), win), rtol=1e-6)
    to_artist = rng.integers(0, 4, 15)
    to_album = rng.integers(0, 6, 15)
    cross = C.precompute_cross_counters(uid, item, ts, lp, like, skip, to_artist, to_album, win)
    assert cross.shape == (n, 9 * len(win))
    for j, other in enumerate((item, to_artist[item], to_album[item])):
        exp = _brute_counts(uid * 100 + other, ts, (lp, like, skip), win)
        for w in range(len(win)):
            np.testing.assert_allclose(cross[:, 9 * w + 3 * j: 9 * w + 3 * j + 3], exp[:, 3 * w: 3 * w + 3],
                                       rtol=1e-6)


# --------------------------------------------------------------------------- event store

def _fake_events(rng, n_users=12, n_items=60, n=1500, days=10):
    uid = rng.integers(1, n_users + 1, n)
    item = rng.integers(1, n_items, n)
    ts = np.sort(rng.integers(0, days * 86400, n))
    etype = rng.choice([0, 0, 0, 0, 1, 2], n)
    played = np.where(etype == 0, rng.integers(0, 101, n), np.nan).astype(np.float32)
    return uid, item, ts, etype, played


def test_event_store_save_load(tmp_path):
    from primus_dlrm_b200.data.dataset import EventStore
    rng = np.random.default_rng(1)
    uid, item, ts, et, pl = _fake_events(rng)
    st = EventStore.from_arrays(uid, item, ts, et, np.nan_to_num(pl), enable_counters=True,
                                item_to_artist=np.arange(60) % 7, item_to_album=np.arange(60) % 11, windows=[1, 7])
    assert st.total_events == uid.size and st.num_users == np.unique(uid).size
    s, e = st.user_slice(int(uid[0]))
    assert (st.flat_uid[s:e] == uid[0]).all() and np.all(np.diff(st.flat_timestamps[s:e]) >= 0)
    assert st.user_counters.shape == (uid.size, 6) and st.cross_counters.shape == (uid.size, 18)
    st.save(tmp_path / "c")
    ld = EventStore.load(tmp_path / "c")
    np.testing.assert_array_equal(ld.flat_item_ids, st.flat_item_ids)
    np.testing.assert_array_equal(ld.cross_counters, st.cross_counters)
    assert not ld.flat_uid.flags.writeable             # shared read-only mapping


def test_event_store_missing_file_raises(tmp_path):
    from primus_dlrm_b200.data.dataset import STORE_ARRAYS, EventStore
    d = tmp_path / "fake_cache"
    d.mkdir()
    for name in STORE_ARRAYS:
        if name != "flat_is_organic":
            np.save(d / f"{name}.npy", np.zeros(8, np.int64))
    (d / "store_meta.json").write_text(json.dumps({"num_users": 1, "total_events": 8, "enable_counters": False,
                                                   "counter_windows_days": []}))
    with pytest.raises(FileNotFoundError, match="flat_is_organic"):
        EventStore.load(d)


# --------------------------------------------------------------------------- preprocessing -> datasets

def _write_raw(root: Path, rng) -> None:
    import pyarrow as pa
    import pyarrow.parquet as pq
    uid, item, ts, et, pl = _fake_events(rng, n=3000, days=12)
    names = np.array(["listen", "like", "dislike"])[et]
    raw = root / "raw" / "50m"
    raw.mkdir(parents=True)
    pq.write_table(pa.table({"uid": uid, "item_id": item, "timestamp": ts, "event_type": names.tolist(),
                             "is_organic": rng.integers(0, 2, uid.size).astype(np.int8),
                             "played_ratio_pct": pl, "track_length_seconds": np.full(uid.size, 200, np.int32)}),
                   raw / "multi_event.parquet", row_group_size=700)
    items = np.arange(60)
    pq.write_table(pa.table({"item_id": items, "artist_id": items % 7}), root / "raw" / "artist_item_mapping.parquet")
    pq.write_table(pa.table({"item_id": items, "album_id": items % 11}), root / "raw" / "album_item_mapping.parquet")
    emb = rng.standard_normal((60, 32)).astype(np.float32)
    pq.write_table(pa.table({"item_id": items, "normalized_embed": [e.tolist() for e in emb]}),
                   root / "raw" / "embeddings.parquet")


def _small_cfg(enable_counters: bool) -> Config:
    cfg = Config.load(CONFIGS / "onetrans_tiny.yaml")
    cfg.data.synthetic.enabled = False
    cfg.data.history_length = 8
    cfg.data.enable_counters = enable_counters
    cfg.data.counter_windows_days = [1, 7]
    cfg.data.use_cache = True
    if enable_counters:
        from primus_dlrm_b200.config import DenseFeatureSpec
        cfg.feature.dense_features += [DenseFeatureSpec("item_counters", 6, project=False),
                                       DenseFeatureSpec("cross_counters", 18, project=True, activation="relu")]
    return cfg


@pytest.fixture(scope="module")
def yambda_root(tmp_path_factory):
    from primus_dlrm_b200.data.preprocessing import preprocess
    root = tmp_path_factory.mktemp("yambda")
    _write_raw(root, np.random.default_rng(5))
    preprocess(root / "raw", root / "processed", "50m", session_gap_seconds=1800, train_days=10, gap_minutes=30,
               test_days=1)
    return root


def test_preprocess_outputs(yambda_root):
    import pyarrow.parquet as pq
    p = yambda_root / "processed"
    meta = json.loads((p / "split_meta.json").read_text())
    assert meta["train_end"] <= meta["test_start"] - 30 * 60
    s = pq.read_table(p / "train_sessions.parquet")
    t = pq.read_table(p / "test_events.parquet")
    n_events = sum(len(x) for x in s.column("item_ids").to_pylist())
    assert n_events == meta["num_train_events"] > 0
    assert t.num_rows == meta["num_test_events"] > 0
    assert set(t.column("uid").to_pylist()) <= set(s.column("uid").to_pylist())
    for ts in s.column("timestamps").to_pylist():
        assert all(b - a <= 1800 for a, b in zip(ts, ts[1:]))   # a session has no gap above the threshold
    pop = np.load(p / "item_popularity.npy")
    assert pop.sum() == meta["num_train_events"]
    assert (yambda_root / "shared_metadata" / "artist_item_mapping.parquet").exists()


@pytest.mark.parametrize("counters", [False, True])
def test_train_dataset_samples(yambda_root, counters):
    from primus_dlrm_b200.data.dataset import (
        LISTEN_PLUS_THRESHOLD, DataPaths, YambdaTrainDataset, collate_to_dict,
    )
    cfg = _small_cfg(counters)
    paths = DataPaths(yambda_root, "50m")
    ds = YambdaTrainDataset(cfg, paths)
    assert len(ds) > 0
    st = ds.store
    for idx in (0, len(ds) // 2, len(ds) - 1):
        s = ds[idx]
        pos = int(ds._positions[idx])
        uid = int(st.flat_uid[pos])
        assert s["uid"] == uid and s["item_id"] == int(st.flat_item_ids[pos])
        assert s["artist_id"] == s["item_id"] % 7 and s["album_id"] == s["item_id"] % 11
        # history = the last L listen+ items strictly before the event, left-padded with 0
        a = max(int(st.user_start[uid]), pos - 500)
        lp_items = st.flat_item_ids[a:pos][st.flat_is_listen_plus[a:pos]][-8:]
        exp = np.zeros(8, np.int64)
        if lp_items.size:
            exp[8 - lp_items.size:] = lp_items
        np.testing.assert_array_equal(s["hist_lp_item_ids"], exp)
        et, pl = int(st.flat_event_types[pos]), float(st.flat_played_ratio[pos])
        assert s["listen_plus"] == float(et == 0 and pl >= LISTEN_PLUS_THRESHOLD)
        if counters:
            assert s["user_counters"].shape == (6,) and s["cross_counters"].shape == (18,)
    batch = collate_to_dict([ds[i] for i in range(16)])
    assert batch["hist_skip_album_ids"].shape == (16, 8) and batch["audio_embed"].dtype == torch.float32
    # the second construction reuses the cache
    cache = paths.cache
    assert any(cache.iterdir())
    ds2 = YambdaTrainDataset(cfg, paths)
    assert len(ds2) == len(ds)


def test_train_dataset_cross_ids(yambda_root):
    from primus_dlrm_b200.data.dataset import DataPaths, YambdaTrainDataset, collate_to_dict
    from primus_dlrm_b200.data.hashing import cross_hash_nway
    cfg = _small_cfg(False)
    cfg.model.cross_features = [CrossFeatureSpec(name="user_x_artist", keys=["uid", "artist_id"], num_embeddings=97),
                                CrossFeatureSpec(name="item_x_hour", keys=["item_id", "hour_of_day"],
                                                 num_embeddings=31, salt=3)]
    cfg.expand_cross_features()
    ds = YambdaTrainDataset(cfg, DataPaths(yambda_root, "50m"))
    s = ds[3]
    assert s["user_x_artist_id"] == cross_hash_nway([s["uid"], s["artist_id"]], 97)
    b = collate_to_dict([ds[i] for i in range(4)])
    assert b["user_x_artist_id"].dtype == torch.int64 and b["item_x_hour_id"].shape == (4,)


def test_eval_dataset(yambda_root):
    from primus_dlrm_b200.data.dataset import DataPaths, YambdaEvalDataset
    cfg = _small_cfg(True)
    ds = YambdaEvalDataset(cfg, DataPaths(yambda_root, "50m"))
    assert len(ds) > 0
    u = ds[0]
    assert "ground_truth_listen_plus" in u and u["history"]["lp_items"].shape == (8,)
    ub = ds.user_batch(u, "cpu")
    assert ub["hist_like_item_ids"].shape == (1, 8) and ub["user_counters"].shape == (1, 6)
    items = np.array([1, 2, 3, 50])
    cb = ds.with_user_features(ds.candidate_batch(items, "cpu"), u, items, "cpu")
    assert cb["item_counters"].shape == (4, 6) and cb["cross_counters"].shape == (4, 18)
    assert ds.get_user_train_items(u["uid"]).size > 0


def test_large_dataset_sampler_partitions():
    from primus_dlrm_b200.data.dataset import LargeDatasetSampler
    data = list(range(103))
    seen = []
    for r in range(4):
        s = LargeDatasetSampler(data, 4, r)
        idx = list(s)
        assert len(idx) == len(s) == 26
        seen += idx
    assert set(seen) == set(range(103))
    s = LargeDatasetSampler(data, 4, 1, shuffle=True, seed=3)
    a = list(s)
    s.set_epoch(1)
    assert list(s) != a and all(0 <= i < 103 for i in a)

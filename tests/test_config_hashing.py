"""Config schema, cross-feature registration, hashing wire format, ranking
metrics and negative samplers (CPU).

Mirrors the reference's ``tests/test_config.py``, ``tests/test_cross_features.py``,
``tests/test_metrics.py`` and ``tests/test_negatives.py``: golden hash values
pin the on-disk wire format (xxhash64 of little-endian int64 keys, mod the
table size), so caches and trained cross tables carry over.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from primus_dlrm_b200.config import (
    Config, CrossFeatureSpec, DataConfig, EmbeddingTableConfig, FeatureConfig, ModelConfig, SchemaConfig,
)

CONFIGS = Path(__file__).resolve().parent.parent / "configs"


# --------------------------------------------------------------------------- config

def test_default_config():
    c = Config()
    assert c.model.model_type in ("dlrm", "onetrans")
    assert c.train.batch_size > 0 and c.train.lr > 0
    assert c.task_names  # default loss weights name at least one task


def test_roundtrip(tmp_path):
    c = Config.load(CONFIGS / "onetrans_tiny.yaml")
    p = tmp_path / "c.yaml"
    c.save(p)
    d = Config.load(p)
    assert d.to_dict() == c.to_dict()


@pytest.mark.parametrize("name", sorted(p.name for p in CONFIGS.glob("*.yaml")))
def test_every_shipped_config_loads(name):
    c = Config.load(CONFIGS / name)
    tables = c.model.resolved_embedding_tables()
    assert tables, name
    for t in tables:
        assert t.embedding_dim > 0 and t.num_embeddings > 0
    # every sequence / scalar feature a table serves is declared
    served = {f for t in tables for f in t.features}
    for f in c.feature.scalar_feature_names:
        assert f in served, (name, f)
    for feats in c.feature.sequence_groups.values():
        for f in feats:
            assert f in served, (name, f)


def test_unknown_key_ignored(tmp_path):
    """Unknown YAML keys are ignored, as the reference's loader does, so
    configs carrying extra keys still load; known keys keep their values."""
    p = tmp_path / "extra.yaml"
    p.write_text("train:\n  batch_sizee: 3\n  batch_size: 7\n")
    c = Config.load(p)
    assert c.train.batch_size == 7


def test_group_lengths_override():
    c = Config.load(CONFIGS / "bench_onetrans_v6_b200.yaml")
    assert c.data.group_length("hist_lp") == 512
    assert c.data.group_length("hist_like") == 128
    assert c.data.group_length("hist_skip") == 256
    assert c.sequence_length_total() == 896


# --------------------------------------------------------------------------- cross features

def _baseline_config() -> Config:
    cfg = Config()
    cfg.model = ModelConfig(model_type="onetrans", embedding_dim=16, embedding_tables=[
        EmbeddingTableConfig("item", ["item"], num_embeddings=100),
        EmbeddingTableConfig("artist", ["artist"], num_embeddings=50),
        EmbeddingTableConfig("album", ["album"], num_embeddings=30),
        EmbeddingTableConfig("uid", ["uid"], num_embeddings=200)])
    cfg.feature = FeatureConfig(scalar_features=["uid", "item", "artist", "album"])
    cfg.data = DataConfig()
    cfg.data.schema = SchemaConfig(batch_to_feature={"item_id": "item", "artist_id": "artist", "album_id": "album"},
                                   kjt_feature_order=["item", "artist", "album", "uid"])
    return cfg


def test_expand_registers_enabled_specs():
    cfg = _baseline_config()
    cfg.model.cross_features = [CrossFeatureSpec(name="user_x_artist", keys=["uid", "artist_id"], num_embeddings=1024),
                                CrossFeatureSpec(name="user_x_hour", keys=["uid", "hour_of_day"], num_embeddings=512)]
    out = cfg.expand_cross_features()
    assert {s.name for s in out} == {"user_x_artist", "user_x_hour"}
    resolved = {t.name: t for t in cfg.model.resolved_embedding_tables()}
    assert resolved["user_x_artist"].embedding_dim == 16
    assert resolved["user_x_hour"].num_embeddings == 512
    assert "user_x_artist" in cfg.feature.scalar_feature_names
    assert cfg.data.schema.batch_to_feature["user_x_hour_id"] == "user_x_hour"
    assert cfg.data.schema.kjt_feature_order[-2:] == ["user_x_artist", "user_x_hour"]


def test_expand_skips_disabled_and_is_idempotent():
    cfg = _baseline_config()
    cfg.model.cross_features = [
        CrossFeatureSpec(name="user_x_artist", keys=["uid", "artist_id"], num_embeddings=1024),
        CrossFeatureSpec(name="user_x_album", keys=["uid", "album_id"], num_embeddings=512, enabled=False)]
    n0 = len(cfg.model.embedding_tables)
    assert len(cfg.expand_cross_features()) == 1
    assert len(cfg.expand_cross_features()) == 0
    assert len(cfg.model.embedding_tables) == n0 + 1
    assert "user_x_album" not in {t.name for t in cfg.model.embedding_tables}
    assert "user_x_album_id" not in cfg.data.schema.batch_to_feature


@pytest.mark.parametrize("spec,match", [
    (CrossFeatureSpec(name="item", keys=["uid", "item_id"], num_embeddings=8), "collides"),
    (CrossFeatureSpec(name="bad", keys=["uid", "nope"], num_embeddings=8), "unknown key"),
    (CrossFeatureSpec(name="z", keys=["uid", "artist_id"], num_embeddings=0), "num_embeddings"),
    (CrossFeatureSpec(name="one", keys=["uid"], num_embeddings=8), "at least 2 keys"),
])
def test_expand_rejects(spec, match):
    cfg = _baseline_config()
    cfg.model.cross_features = [spec]
    with pytest.raises(ValueError, match=match):
        cfg.expand_cross_features()


def test_expand_spec_order_and_3way():
    cfg = _baseline_config()
    cfg.model.cross_features = [
        CrossFeatureSpec(name="z_first", keys=["uid", "artist_id"], num_embeddings=8),
        CrossFeatureSpec(name="a_second", keys=["uid", "album_id", "hour_of_day"], num_embeddings=8)]
    cfg.expand_cross_features()
    assert cfg.feature.scalar_feature_names[-2:] == ["z_first", "a_second"]


# --------------------------------------------------------------------------- hashing

def test_cross_hash_golden_vectors():
    from primus_dlrm_b200.data.hashing import cross_hash_int64
    assert cross_hash_int64(1, 2, 1000) == 524
    assert cross_hash_int64(1, 2, 1 << 30) == 1056167084
    assert cross_hash_int64(42, 7, 1_000_000) == 924376
    assert cross_hash_int64(0, 0, 1000) == 434
    assert cross_hash_int64(-1, -1, 1000) == 28


def test_cross_hash_nway_golden_vectors():
    from primus_dlrm_b200.data.hashing import cross_hash_nway
    assert cross_hash_nway([1, 2, 3], 1000) == 706
    assert cross_hash_nway([1, 2, 3], 1 << 30) == 633392634
    assert cross_hash_nway([42, 7, 15], 1_000_000) == 847584
    assert cross_hash_nway([1, 2, 3, 4], 1000) == 45
    assert cross_hash_nway([3, 2, 1], 1000) == 313
    with pytest.raises(AssertionError):
        cross_hash_nway([1], 1000)


def test_numpy_xxh64_matches_scalar_path():
    """The vectorised numpy XXH64 gives the same digests as the scalar path."""
    from primus_dlrm_b200.data.hashing import cross_hash_batch, cross_hash_int64, xxh64_np
    a = np.array([1, 42, 100, 0, -1, 1 << 40], dtype=np.int64)
    b = np.array([2, 7, 200, 0, -1, 1 << 30], dtype=np.int64)
    for salt in (0, 5):
        exp = np.array([cross_hash_int64(int(x), int(y), 12345, salt) for x, y in zip(a, b)])
        np.testing.assert_array_equal(cross_hash_batch(a, b, 12345, salt), exp)
    # broadcast of a scalar operand
    got = cross_hash_batch(np.array([1, 2, 3]), np.array([7]), 1000)
    np.testing.assert_array_equal(got, [cross_hash_int64(i, 7, 1000) for i in (1, 2, 3)])
    # 3 keys through the numpy kernel (first-lane path) match the n-way digest
    from primus_dlrm_b200.data.hashing import cross_hash_nway
    w = np.array([[1, 2, 3]], dtype="<u8")
    assert int(xxh64_np(w, 0)[0]) % 1000 == cross_hash_nway([1, 2, 3], 1000)


def test_cross_hash_range_salt_asymmetry():
    from primus_dlrm_b200.data.hashing import cross_hash_int64
    for t in (1, 7, 1024, 1_000_000):
        for a, b in [(0, 0), (1, 2), (123, 456), (1 << 40, 1 << 30)]:
            assert 0 <= cross_hash_int64(a, b, t) < t
    assert cross_hash_int64(1, 2, 1000) != cross_hash_int64(2, 1, 1000)
    assert cross_hash_int64(1, 2, 1000, salt=0) != cross_hash_int64(1, 2, 1000, salt=5)


# --------------------------------------------------------------------------- metrics

def test_ndcg_recall():
    from primus_dlrm_b200.evaluation.metrics import metrics_from_ranking, ndcg_at_k, recall_at_k
    assert ndcg_at_k([(0, 10.0), (1, 9.0), (2, 8.0)], {0, 1, 2}, 3) == pytest.approx(1.0)
    exp = (1.0 / np.log2(4)) / (1.0 / np.log2(2))
    assert ndcg_at_k([(3, 10.0), (4, 9.0), (0, 8.0)], {0}, 3) == pytest.approx(exp)
    assert ndcg_at_k([(0, 10.0)], set(), 3) == 0.0
    assert recall_at_k([(0, 10.0), (1, 9.0), (2, 8.0)], {0, 1}, 3) == pytest.approx(1.0)
    assert recall_at_k([(3, 10.0), (4, 9.0), (0, 8.0)], {0, 1}, 3) == pytest.approx(0.5)
    assert recall_at_k([(0, 1.0)], set(), 3) == 0.0
    # dict input is ranked by score
    assert ndcg_at_k({5: 0.1, 6: 0.9}, {6}, 1) == pytest.approx(1.0)
    m = metrics_from_ranking(np.array([3, 4, 0]), {0}, [1, 3])
    assert m["recall@1"] == 0.0 and m["recall@3"] == 1.0 and m["ndcg@3"] == pytest.approx(exp)


# --------------------------------------------------------------------------- negatives

def test_negative_samplers():
    from primus_dlrm_b200.data.negatives import MixedSampler, PopularitySampler, UniformSampler
    negs = UniformSampler(1000, seed=42).sample(10)
    assert len(negs) == 10 and len(set(negs.tolist())) == 10 and all(0 <= n < 1000 for n in negs)
    ex = {0, 1, 2, 3, 4}
    negs = UniformSampler(100, seed=42).sample(5, exclude=ex)
    assert len(negs) == 5 and not (set(negs.tolist()) & ex)
    counts = np.ones(100, np.int64)
    counts[0] = 1000
    assert 0 in PopularitySampler(100, counts, seed=42).sample(50).tolist()
    assert len(MixedSampler(100, np.ones(100, np.int64), uniform_ratio=0.5, seed=42).sample(10)) == 10

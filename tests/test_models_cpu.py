"""Model forward/backward on CPU (the eager path of every op): OneTrans with
and without the pyramid, counters, cross features; DLRM two-tower with each
interaction (concat MLP, dot, DCNv2 full and low-rank) and the Criteo
layout; fused heads+loss against ``MultiTaskLoss``; contrastive cross scores;
analytic FLOPs.  Coverage follows the reference's ``tests/test_model.py``.
"""
from __future__ import annotations

import copy
from pathlib import Path

import pytest
import torch

from primus_dlrm_b200.config import (
    Config, CrossFeatureSpec, DenseFeatureSpec, EmbeddingTableConfig, FeatureConfig, ModelConfig, SchemaConfig,
    TransformerConfig,
)
from primus_dlrm_b200.models.dlrm import DLRMBaseline
from primus_dlrm_b200.models.onetrans import OneTransModel, pyramid_schedule
from primus_dlrm_b200.training.losses import InBatchBPRLoss, MultiTaskLoss

CONFIGS = Path(__file__).resolve().parent.parent / "configs"
SIZES = {"item": 100, "artist": 50, "album": 30, "uid": 200}
POOLS = ("lp", "like", "skip")


def _schema() -> SchemaConfig:
    b2f = {"item_id": "item", "artist_id": "artist", "album_id": "album"}
    for p in POOLS:
        for k in ("item", "artist", "album"):
            b2f[f"hist_{p}_{k}_ids"] = f"hist_{p}_{k}"
    return SchemaConfig(batch_to_feature=b2f)


def _features(counter_windows: int = 0) -> FeatureConfig:
    dense = [DenseFeatureSpec("audio_embed", 32, project=True, activation="gelu")]
    if counter_windows:
        W = counter_windows
        dense += [DenseFeatureSpec("user_counters", 3 * W, project=False, tower="user"),
                  DenseFeatureSpec("item_counters", 3 * W, project=False, tower="item"),
                  DenseFeatureSpec("cross_counters", 9 * W, project=True, activation="relu")]
    fc = FeatureConfig(sequence_groups={f"hist_{p}": [f"hist_{p}_{k}" for k in ("item", "artist", "album")]
                                        for p in POOLS},
                       scalar_features=["uid", "item", "artist", "album"], dense_features=dense)
    for s in fc.scalar_features:
        s.tower = "user" if s.name == "uid" else "item"
    return fc


def _batch(B=4, L=10, windows=0, cross: dict | None = None, seed=0):
    g = torch.Generator().manual_seed(seed)
    b = {}
    for p in POOLS:
        for k in ("item", "artist", "album"):
            b[f"hist_{p}_{k}_ids"] = torch.randint(0, SIZES[k], (B, L), generator=g)
    b["uid"] = torch.randint(0, 200, (B,), generator=g)
    for k in ("item", "artist", "album"):
        b[f"{k}_id"] = torch.randint(0, SIZES[k], (B,), generator=g)
    b["audio_embed"] = torch.randn(B, 32, generator=g)
    for t in ("listen_plus", "like", "dislike"):
        b[t] = torch.randint(0, 2, (B,), generator=g).float()
    b["listen_pct"] = torch.rand(B, generator=g)
    if windows:
        b["user_counters"] = torch.rand(B, 3 * windows, generator=g)
        b["item_counters"] = torch.rand(B, 3 * windows, generator=g)
        b["cross_counters"] = torch.rand(B, 9 * windows, generator=g)
    for name, n in (cross or {}).items():
        b[f"{name}_id"] = torch.randint(0, n, (B,), generator=g)
    return b


def _config(model_type: str, tasks=("listen_plus",), windows=0, L=10, **model_kw) -> Config:
    c = Config()
    c.data.history_length = L
    c.data.schema = _schema()
    c.feature = _features(windows)
    c.data.enable_counters = windows > 0
    c.data.counter_windows_days = list(range(1, windows + 1))
    if model_type == "onetrans":
        tables = [EmbeddingTableConfig(k, [k] + [f"hist_{p}_{k}" for p in POOLS], num_embeddings=n)
                  for k, n in SIZES.items() if k != "uid"] + [EmbeddingTableConfig("uid", ["uid"], 200)]
        tr = TransformerConfig(d_model=32, n_heads=4, n_layers=2, ffn_mult=2, n_ns_tokens=4, dropout=0.0,
                               attention_impl="sdpa", **model_kw.pop("transformer", {}))
        c.model = ModelConfig(model_type="onetrans", embedding_dim=16, embedding_tables=tables, transformer=tr,
                              **model_kw)
    else:
        tables = []
        for k in ("item", "artist", "album"):
            tables.append(EmbeddingTableConfig(f"hist_{k}", [f"hist_{p}_{k}" for p in POOLS], SIZES[k],
                                               pooling="mean"))
            tables.append(EmbeddingTableConfig(k, [k], SIZES[k]))
        tables.append(EmbeddingTableConfig("uid", ["uid"], 200))
        kw = dict(embedding_dim=16, top_mlp_dims=[32, 16], bottom_mlp_dims=[32])
        kw.update(model_kw)
        c.model = ModelConfig(model_type="dlrm", embedding_tables=tables, **kw)
    c.train.loss_weights = {t: 1.0 for t in tasks}
    c.train.regression_tasks = ["listen_pct"] if "listen_pct" in tasks else []
    return c


def _grads_ok(model) -> None:
    n = 0
    for name, p in model.named_parameters():
        if p.grad is not None:
            assert torch.isfinite(p.grad).all(), name
            n += 1
    assert n > 0


# --------------------------------------------------------------------------- DLRM

@pytest.mark.parametrize("interaction,kw", [("concat_mlp", {}), ("dot", {}), ("dcnv2", {}),
                                            ("dcnv2", {"dcn_low_rank": 8})])
def test_dlrm_forward_backward(interaction, kw):
    cfg = _config("dlrm", tasks=("listen_plus", "like"), interaction_type=interaction, **kw)
    model = DLRMBaseline(cfg)
    out = model(_batch())
    assert set(out) == {"listen_plus", "like"} and out["like"].shape == (4,)
    total, per = MultiTaskLoss(cfg.train.loss_weights)(out, _batch())
    total.backward()
    _grads_ok(model)


def test_dlrm_low_rank_cross_has_fewer_params():
    full = DLRMBaseline(_config("dlrm", interaction_type="dcnv2"))
    low = DLRMBaseline(_config("dlrm", interaction_type="dcnv2", dcn_low_rank=4))
    n = lambda m: sum(p.numel() for p in m.interaction.parameters())  # noqa: E731
    assert n(low) < n(full)


@pytest.mark.parametrize("interaction", ["concat_mlp", "dot"])
def test_dlrm_with_counters(interaction):
    cfg = _config("dlrm", windows=2, interaction_type=interaction)
    model = DLRMBaseline(cfg)
    out = model(_batch(windows=2))
    out["listen_plus"].sum().backward()
    _grads_ok(model)


def test_dlrm_criteo_layout():
    cfg = Config.load(CONFIGS / "bench_dlrm_dcnv2_b200.yaml")
    for t in cfg.model.embedding_tables:
        t.num_embeddings = min(t.num_embeddings, 1000)
    cfg.model.dcn_low_rank = 16
    cfg.model.top_mlp_dims = [64, 32]
    cfg.model.bottom_mlp_dims = [32, 16]
    cfg.model.embedding_dim = 16
    from primus_dlrm_b200.data.synthetic import generate_batch
    b = generate_batch(cfg, 8, seed=1)
    model = DLRMBaseline(cfg)
    total, per, logits = model.forward_loss(b, cfg.train.loss_weights, cfg.train.regression_tasks)
    assert logits["label"].shape == (8,)
    total.backward()
    _grads_ok(model)


def test_dlrm_cross_scores_diagonal_matches_predictions():
    cfg = _config("dlrm")
    model = DLRMBaseline(cfg).eval()
    b = _batch(B=5)
    with torch.no_grad():
        preds, cross = model.forward_with_cross_scores(b)
    assert cross.shape == (5, 5)
    torch.testing.assert_close(cross.diagonal(), preds["listen_plus"], rtol=1e-5, atol=1e-5)


# --------------------------------------------------------------------------- OneTrans

def test_pyramid_schedule():
    s = pyramid_schedule(300, 8, 4)
    assert s[0] == 300 and s[-1] == 8
    assert all(a >= b for a, b in zip(s, s[1:]))
    assert pyramid_schedule(896, 16, 8)[-1] == 16


@pytest.mark.parametrize("pyramid", [True, False])
def test_onetrans_forward_backward(pyramid):
    cfg = _config("onetrans", tasks=("listen_plus", "like", "listen_pct"), transformer={"use_pyramid": pyramid})
    model = OneTransModel(cfg)
    b = _batch()
    out = model(b)
    assert all(v.shape == (4,) for v in out.values())
    total, per, logits = model.forward_loss(b, cfg.train.loss_weights, cfg.train.regression_tasks)
    # fused heads + loss equals the unfused multi-task loss
    ref_total, ref_per = MultiTaskLoss(cfg.train.loss_weights, cfg.train.regression_tasks)(out, b)
    torch.testing.assert_close(total, ref_total, rtol=1e-5, atol=1e-6)
    for t in per:
        torch.testing.assert_close(per[t], ref_per[t], rtol=1e-5, atol=1e-6)
    total.backward()
    _grads_ok(model)
    assert not torch.isnan(total)


def test_onetrans_counters_and_cross_features():
    cfg = _config("onetrans", windows=2)
    cfg.model.cross_features = [CrossFeatureSpec(name="user_x_artist", keys=["uid", "artist_id"], num_embeddings=64)]
    cfg.expand_cross_features()
    model = OneTransModel(cfg)
    t = [t for t in model.emb.tables() if t.name == "user_x_artist"][0]
    w0 = t.weight.detach().clone()
    out = model(_batch(windows=2, cross={"user_x_artist": 64}))
    out["listen_plus"].sum().backward()
    # the sparse optimizer update runs inside the lookup's backward
    assert not torch.equal(t.weight.detach(), w0)
    _grads_ok(model)


def test_onetrans_cross_scores_and_bpr():
    cfg = _config("onetrans")
    model = OneTransModel(cfg)
    b = _batch(B=6)
    preds, cross = model.forward_with_cross_scores(b)
    assert cross.shape == (6, 6)
    loss = InBatchBPRLoss()(cross, b["listen_plus"])
    assert torch.isfinite(loss)
    (loss + preds["listen_plus"].sum()).backward()
    _grads_ok(model)


def test_onetrans_deterministic_in_seed():
    cfg = _config("onetrans")
    torch.manual_seed(0)
    a = OneTransModel(cfg)
    torch.manual_seed(0)
    b = OneTransModel(copy.deepcopy(cfg))
    x = _batch()
    torch.testing.assert_close(a(x)["listen_plus"], b(x)["listen_plus"])


def test_onetrans_flops_per_sample():
    cfg = Config.load(CONFIGS / "bench_onetrans_v6_b200.yaml")
    m = OneTransModel(cfg, meta_device=True, device="meta")
    gf = m.get_num_flops_per_sample() / 1e9
    assert 20 < gf < 40, gf
    # the FLOP count grows with depth
    cfg.model.transformer.n_layers = 4
    assert OneTransModel(cfg, meta_device=True, device="meta").get_num_flops_per_sample() / 1e9 < gf


def test_bpr_loss_value():
    s = torch.tensor([[2.0, 0.0], [1.0, 1.0]])
    y = torch.tensor([1.0, 0.0])
    exp = -torch.nn.functional.logsigmoid(torch.tensor((2.0 - 0.0) / 0.1))
    torch.testing.assert_close(InBatchBPRLoss(0.1)(s, y), exp)


@pytest.mark.parametrize("pyramid", [True, False])
def test_onetrans_kv_cached_scoring_is_exact(pyramid):
    """score_candidates (S stream once, NS tokens per candidate) == forward on
    (user history, candidate) rows."""
    cfg = _config("onetrans", windows=2, transformer={"use_pyramid": pyramid})
    torch.manual_seed(0)
    model = OneTransModel(cfg).eval()
    full = _batch(B=7, windows=2, seed=5)
    user_keys = [k for k in full if k.startswith("hist_")] + ["uid", "user_counters"]
    user = {k: full[k][:1] for k in user_keys}
    cand = {k: full[k] for k in ("item_id", "artist_id", "album_id", "audio_embed", "item_counters",
                                 "cross_counters")}
    rows = dict(cand)
    for k in user_keys:
        rows[k] = user[k].expand(7, *user[k].shape[1:])
    with torch.no_grad():
        ref = model(rows)["listen_plus"]
        got = model.score_candidates(user, cand, "listen_plus", batch_size=3)
    torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-5)


def test_ranking_eval_uses_kv_cache():
    from primus_dlrm_b200.data.dataset import SyntheticEvalDataset
    from primus_dlrm_b200.evaluation.metrics import score_candidates
    cfg = Config.load(CONFIGS / "onetrans_tiny.yaml")
    cfg.data.history_length = 6
    model = OneTransModel(cfg).eval()
    ds = SyntheticEvalDataset(cfg, num_users=2, num_items_with_history=30)
    s = ds[0]
    items = torch.arange(9).numpy()
    ub = ds.user_batch(s, "cpu")
    cb = ds.with_user_features(ds.candidate_batch(items, "cpu"), s, items, "cpu")
    got = score_candidates(model, ub, cb, "listen_plus")
    rows = dict(cb)
    for k, v in ub.items():
        rows[k] = v.expand(len(items), *v.shape[1:])
    with torch.no_grad():
        ref = model(rows)["listen_plus"]
    torch.testing.assert_close(got, ref.float(), rtol=1e-4, atol=1e-5)

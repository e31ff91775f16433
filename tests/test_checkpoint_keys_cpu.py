"""The model's state_dict keys and shapes are the reference's checkpoint
contract: a .pt written by either framework loads into the other with strict
load_state_dict. The expected map is rebuilt here from the config with the
reference's module-construction rules (primus_dlrm/models/onetrans.py:279-390:
TorchRec EmbeddingCollection ``emb.ec.embeddings.<table>``, per-group
SequentialTokenizer ``proj.{0,2}`` + ``pos_emb`` [2048, D], ``dense_projs``
for projected dense features, AutoSplitTokenizer, MixedAttention /
MixedFFN blocks, final RMSNorm, head bridge, task heads, contrastive heads)."""
from pathlib import Path

import torch

from primus_dlrm_b200.config import Config
from primus_dlrm_b200.models.onetrans import OneTransModel

CONFIGS = Path(__file__).resolve().parent.parent / "configs"


def _expected_onetrans(cfg) -> dict[str, tuple[int, ...]]:
    mc, fc, ot = cfg.model, cfg.feature, cfg.model.transformer
    D, E, NS = ot.d_model, mc.embedding_dim, ot.n_ns_tokens
    F = D * ot.ffn_mult
    exp: dict[str, tuple[int, ...]] = {}
    for t in mc.resolved_embedding_tables():
        exp[f"emb.ec.embeddings.{t.name}.weight"] = (t.num_embeddings, t.embedding_dim or E)
    for g, feats in fc.sequence_groups.items():
        exp[f"seq_tokenizers.{g}.proj.0.weight"] = (D, len(feats) * E)
        exp[f"seq_tokenizers.{g}.proj.0.bias"] = (D,)
        exp[f"seq_tokenizers.{g}.proj.2.weight"] = (D, D)
        exp[f"seq_tokenizers.{g}.proj.2.bias"] = (D,)
        if ot.pos_embed:
            exp[f"seq_tokenizers.{g}.pos_emb.weight"] = (2048, D)
    ns_raw = len(fc.scalar_feature_names) * E
    for df in fc.dense_features:
        if df.project:
            exp[f"dense_projs.{df.name}.0.weight"] = (E, df.dim)
            exp[f"dense_projs.{df.name}.0.bias"] = (E,)
            ns_raw += E
        else:
            ns_raw += df.dim
    exp["ns_tokenizer.proj.0.weight"] = (NS * D, ns_raw)
    exp["ns_tokenizer.proj.0.bias"] = (NS * D,)
    exp["ns_tokenizer.proj.2.weight"] = (NS * D, NS * D)
    exp["ns_tokenizer.proj.2.bias"] = (NS * D,)
    for i in range(ot.n_layers):
        b = f"blocks.{i}"
        exp[f"{b}.norm1.weight"] = (D,)
        exp[f"{b}.attn.s_qkv.weight"] = (3 * D, D)
        exp[f"{b}.attn.ns_qkv_weight"] = (NS, 3 * D, D)
        exp[f"{b}.attn.out_proj.weight"] = (D, D)
        exp[f"{b}.norm2.weight"] = (D,)
        exp[f"{b}.ffn.s_w1.weight"] = (F, D)
        exp[f"{b}.ffn.s_w2.weight"] = (D, F)
        exp[f"{b}.ffn.ns_w1"] = (NS, F, D)
        exp[f"{b}.ffn.ns_w2"] = (NS, D, F)
    exp["final_norm.weight"] = (D,)
    exp["head_proj.0.weight"] = (D, NS * D)
    exp["head_proj.0.bias"] = (D,)
    for task in cfg.task_names:
        exp[f"heads.{task}.weight"] = (1, D)
        exp[f"heads.{task}.bias"] = (1,)
    exp["contrastive_user_proj.weight"] = (D, D)
    exp["contrastive_user_proj.bias"] = (D,)
    n_item = len([sf for sf in fc.item_scalar_features])
    exp["contrastive_item_proj.0.weight"] = (D, n_item * E)
    exp["contrastive_item_proj.0.bias"] = (D,)
    return exp


def _check(cfg):
    model = OneTransModel(cfg)
    got = {k: tuple(v.shape) for k, v in model.state_dict().items()}
    exp = _expected_onetrans(cfg)
    assert set(got) == set(exp), (f"missing {sorted(set(exp) - set(got))}, "
                                  f"unexpected {sorted(set(got) - set(exp))}")
    bad = {k: (got[k], exp[k]) for k in exp if got[k] != exp[k]}
    assert not bad, f"shape mismatch: {bad}"
    for k, v in model.state_dict().items():
        assert v.dtype == torch.float32, f"{k} is {v.dtype}; checkpoints hold fp32"


def test_onetrans_state_dict_matches_reference_layout_tiny():
    _check(Config.load(CONFIGS / "onetrans_tiny.yaml"))


def test_onetrans_state_dict_matches_reference_layout_v6_shapes_small_tables():
    cfg = Config.load(CONFIGS / "bench_onetrans_v6_b200.yaml")
    for t in cfg.model.embedding_tables:      # keep the CPU test small; shapes follow the config
        t.num_embeddings = 1000
    _check(cfg)


def test_compiled_block_prefix_is_canonicalised_on_load():
    """Reference checkpoints of torch.compile'd runs carry ``blocks.<i>._orig_mod.``
    (primus_dlrm/models/onetrans.py:382-390); loading strips it."""
    from primus_dlrm_b200.parallel.state import _canonical
    cfg = Config.load(CONFIGS / "onetrans_tiny.yaml")
    model = OneTransModel(cfg)
    sd = model.state_dict()
    compiled = {(k.replace("blocks.0.", "blocks.0._orig_mod.") if k.startswith("blocks.0.") else k): v
                for k, v in sd.items()}
    fixed = {_canonical(k): v for k, v in compiled.items()}
    model.load_state_dict(fixed, strict=True)

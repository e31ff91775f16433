"""DLRM models.

``DLRMBaseline`` (``dlrm_layout: two_tower``, the reference DLRM++,
``primus_dlrm/models/dlrm.py``): user tower = user scalars + mean-pooled
sequence features + raw user dense -> bottom MLP; item tower = item scalars
+ projected dense + raw item dense -> bottom MLP; interaction over
[user] x [item (+ ReLU-projected cross counters)]; one head per task.

``dlrm_layout: criteo`` (the DLRM-DCNv2 benchmark config, additive): all dense
features -> bottom MLP; every scalar (single-id) sparse feature is one
embedding; interaction over [bottom-MLP output] x [embeddings]; heads.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from primus_dlrm_b200.config import Config
from primus_dlrm_b200.models.base import BaseModel
from primus_dlrm_b200.models.embedding import Embeddings
from primus_dlrm_b200.models.heads import fused_heads_loss
from primus_dlrm_b200.models.interaction import build_interaction, make_mlp
from primus_dlrm_b200.ops.embedding import SparseOptimizer
from primus_dlrm_b200.ops.mlp import mlp_chain


class DLRMBaseline(BaseModel):
    def __init__(self, config: Config, device: torch.device | None = None, meta_device: bool = False):
        super().__init__()
        self.config = config
        mc, fc, tc = config.model, config.feature, config.train
        self.tasks = list(config.task_names)
        self.layout = mc.dlrm_layout
        D = mc.embedding_dim
        device = torch.device("cpu") if device is None else torch.device(device)
        emb_device = torch.device("meta") if meta_device else device
        opt = SparseOptimizer(kind=tc.embedding_optimizer, lr=tc.embedding_lr, eps=tc.embedding_eps,
                              weight_decay=tc.weight_decay)
        self.emb = Embeddings(mc.resolved_embedding_tables(), device=emb_device, embedding_init=mc.embedding_init,
                              scalar_feature_names=set(fc.scalar_feature_names), optimizer=opt)
        self.dense_projs = nn.ModuleDict()
        if self.layout == "criteo":
            dense_dim = sum(df.dim for df in fc.dense_features)
            self.bottom_mlp = make_mlp([dense_dim] + mc.bottom_mlp_dims, mc.dropout).to(device)
            bot = mc.bottom_mlp_dims[-1] if mc.bottom_mlp_dims else dense_dim
            emb_dims = [self.emb.feature_dim(f) for f in fc.scalar_feature_names]
            self.interaction = build_interaction(mc.interaction_type, [bot], emb_dims, mc.top_mlp_dims,
                                                 mc.dcn_num_cross_layers, mc.dropout, mc.dcn_low_rank).to(device)
        else:
            for df in fc.dense_features:
                if df.project:
                    act = nn.ReLU(inplace=True) if df.activation == "relu" else nn.GELU()
                    self.dense_projs[df.name] = nn.Sequential(nn.Linear(df.dim, D, device=device), act)
            n_seq = sum(self.emb.feature_dim(f) for feats in fc.sequence_groups.values() for f in feats)
            n_user_raw = sum(df.dim for df in fc.dense_features if not df.project and df.in_user_tower())
            user_dim = sum(self.emb.feature_dim(s.name) for s in fc.user_scalar_features) + n_seq + n_user_raw
            if mc.bottom_mlp_dims:
                self.user_bottom_mlp = make_mlp([user_dim] + mc.bottom_mlp_dims, mc.dropout).to(device)
                user_out = mc.bottom_mlp_dims[-1]
            else:
                self.user_bottom_mlp, user_out = nn.Identity(), user_dim
            n_proj = sum(1 for df in fc.dense_features if df.project)
            n_item_raw = sum(df.dim for df in fc.dense_features if not df.project and df.in_item_tower())
            item_dim = sum(self.emb.feature_dim(s.name) for s in fc.item_scalar_features) + n_proj * D + n_item_raw
            if mc.bottom_mlp_dims:
                self.item_bottom_mlp = make_mlp([item_dim] + mc.bottom_mlp_dims, mc.dropout).to(device)
                item_out = mc.bottom_mlp_dims[-1]
            else:
                self.item_bottom_mlp, item_out = nn.Identity(), item_dim
            item_dims = [item_out]
            if any(df.project and df.activation == "relu" for df in fc.dense_features):
                item_dims.append(D)
            self.interaction = build_interaction(mc.interaction_type, [user_out], item_dims, mc.top_mlp_dims,
                                                 mc.dcn_num_cross_layers, mc.dropout, mc.dcn_low_rank).to(device)
        self.heads = nn.ModuleDict({t: nn.Linear(self.interaction.output_dim, 1, device=device)
                                    for t in self.tasks})

    # ------------------------------------------------------------------
    def get_num_flops_per_sample(self) -> float:
        """Analytic fwd+bwd FLOPs per sample: 6 per multiply-accumulate of every
        dense projection (Linear layers, the DCNv2 cross factors); lookups and
        elementwise work are not counted (as in the OneTrans estimator)."""
        fl = 0
        for name, m in self.named_modules():
            if isinstance(m, nn.Linear) and not name.startswith("emb"):
                fl += 6 * m.in_features * m.out_features
        inter = self.interaction
        for attr in ("cross_u", "cross_v", "cross_weights"):
            for p in getattr(inter, attr, []):
                fl += 6 * p.numel()
        return float(fl)

    def _dtype(self) -> torch.dtype:
        return torch.bfloat16 if (torch.is_autocast_enabled("cuda") or torch.is_autocast_enabled("cpu")) \
            else torch.float32

    def _embs(self, batch: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
        f2k = self.config.feature_to_batch_key()
        names = [f for f in self.config.feature.all_ec_feature_names() if f2k.get(f, f) in batch]
        feats = {f: batch[f2k.get(f, f)] for f in names}
        offs = {}
        for f in names:
            lk = f2k.get(f, f) + "__lengths"
            if lk in batch and self.emb.is_pooled(f):
                lens = batch[lk].long()
                offs[f] = torch.cat([lens.new_zeros(1), lens.cumsum(0)])
        outs = self.emb.lookup_groups(feats, [[f] for f in names], dtype=self._dtype(), offsets=offs or None)
        return dict(zip(names, outs))

    def _towers(self, batch):
        fc = self.config.feature
        embs = self._embs(batch)
        if self.layout == "criteo":
            dense = torch.cat([batch[df.name].float() for df in fc.dense_features], dim=-1)
            if torch.is_autocast_enabled("cuda") and dense.is_cuda:
                dense = dense.to(torch.bfloat16)
            bottom = mlp_chain(self.bottom_mlp, dense)
            return [bottom], [embs[f] for f in fc.scalar_feature_names]
        up = [embs[s.name] for s in fc.user_scalar_features]
        for feats in fc.sequence_groups.values():
            up.extend(embs[f] for f in feats)
        up.extend(batch[df.name] for df in fc.dense_features if not df.project and df.in_user_tower())
        user = mlp_chain(self.user_bottom_mlp, torch.cat([p.to(up[0].dtype) for p in up], dim=-1))
        ip = [embs[s.name] for s in fc.item_scalar_features]
        ip.extend(self.dense_projs[df.name](batch[df.name]) for df in fc.dense_features if df.project)
        ip.extend(batch[df.name] for df in fc.dense_features if not df.project and df.in_item_tower())
        item = mlp_chain(self.item_bottom_mlp, torch.cat([p.to(ip[0].dtype) for p in ip], dim=-1))
        items = [item]
        for df in fc.dense_features:
            if df.project and df.activation == "relu":
                items.append(self.dense_projs[df.name](batch[df.name]))
                break
        return [user], items

    def forward(self, batch: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
        u, i = self._towers(batch)
        h = self.interaction(user_features=u, item_features=i)
        return {t: head(h).squeeze(-1) for t, head in self.heads.items()}

    def forward_loss(self, batch, loss_weights, regression_tasks):
        u, i = self._towers(batch)
        h = self.interaction(user_features=u, item_features=i)
        return fused_heads_loss(self.heads, h, batch, loss_weights, regression_tasks)

    def forward_with_cross_scores(self, batch, cross_task: str = ""):
        u, i = self._towers(batch)
        h = self.interaction(user_features=u, item_features=i)
        preds = {t: head(h).squeeze(-1) for t, head in self.heads.items()}
        user, item = u[0], i[0]
        B = user.shape[0]
        ue = user.unsqueeze(1).expand(B, B, -1).reshape(B * B, -1)
        ie = [item.unsqueeze(0).expand(B, B, -1).reshape(B * B, -1)]
        ie += [torch.zeros(B * B, x.shape[-1], device=x.device, dtype=x.dtype) for x in i[1:]]
        task = cross_task or self.tasks[0]
        cross = self.heads[task](self.interaction(user_features=[ue], item_features=ie)).squeeze(-1).view(B, B)
        return preds, cross

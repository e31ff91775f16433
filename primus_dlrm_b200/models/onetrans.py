"""OneTrans: one causal Transformer over behaviour-sequence (S) and
non-sequential (NS) tokens.

Architecture and parameter layout follow ``primus_dlrm/models/onetrans.py``
(so checkpoints interchange key-for-key):

* per-group ``SequentialTokenizer`` (Linear(G*E, D) -> GELU -> Linear(D, D)
  + learned positions) builds the S tokens (``onetrans.py:238-257``);
* ``AutoSplitTokenizer`` maps the concatenated NS features to ``n_ns`` tokens
  (``onetrans.py:260-276``);
* blocks use *mixed parameterisation*: S tokens share ``s_qkv`` / ``s_w1`` /
  ``s_w2``, each NS token has its own slice of ``ns_qkv_weight`` /
  ``ns_w1`` / ``ns_w2`` (``onetrans.py:85-204``);
* pyramid query pruning: layer ``l`` keeps the last ``schedule[l] + n_ns``
  queries and attends bottom-right causally (``onetrans.py:50-67``).

Execution (B200): the lookup writes every pool's ``[B, L, 3E]`` tokenizer
input in bf16 with one kernel; the S and NS projections write into one
``[B, T, 3D]`` QKV buffer (no concatenation); norm kernels fuse the
attention residual; heads + multi-task loss are one fused op.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from primus_dlrm_b200.config import Config
from primus_dlrm_b200.models.base import BaseModel
from primus_dlrm_b200.models.embedding import Embeddings
from primus_dlrm_b200.models.heads import fused_heads_loss
from primus_dlrm_b200.ops import dense
from primus_dlrm_b200.ops.attention import (
    _native_ok as _fmha_native_ok, causal_attention_all_rows, pyramid_attention, pyramid_attention_qkv,
)
from primus_dlrm_b200.ops.embedding import SparseOptimizer
from primus_dlrm_b200.ops.norm import add_norm, make_norm, norm_with_tail


def pyramid_schedule(l_s: int, l_ns: int, n_layers: int) -> list[int]:
    """S-token query count per layer, shrinking linearly from ``l_s`` to
    ``l_ns`` (rounded, floored at ``l_ns``; one layer keeps ``l_ns``)."""
    if n_layers <= 1:
        return [l_ns]
    step = (l_s - l_ns) / (n_layers - 1)
    return [max(int(round(l_s - i * step)), l_ns) for i in range(n_layers)]


def _xavier_per_token(w: torch.Tensor) -> None:
    for i in range(w.shape[0]):
        nn.init.xavier_uniform_(w.data[i])


class MixedAttention(nn.Module):
    def __init__(self, d_model: int, n_heads: int, n_ns_tokens: int, dropout: float = 0.0,
                 attention_impl: str = "sdpa"):
        super().__init__()
        if d_model % n_heads:
            raise ValueError("d_model must be divisible by n_heads")
        if attention_impl not in ("sdpa", "fav2", "fav4", "turbo", "native", "mask"):
            raise ValueError(f"Unknown attention_impl: {attention_impl!r}. "
                             f"Supported: 'sdpa', 'fav2', 'fav4', 'turbo', 'native'")
        self.d_model = d_model
        self.n_heads = n_heads
        self.d_head = d_model // n_heads
        self.n_ns = n_ns_tokens
        self.attention_impl = attention_impl
        self.s_qkv = nn.Linear(d_model, 3 * d_model, bias=False)
        self.ns_qkv_weight = nn.Parameter(torch.empty(n_ns_tokens, 3 * d_model, d_model))
        self.out_proj = nn.Linear(d_model, d_model, bias=False)
        self.attn_drop = dropout
        nn.init.xavier_uniform_(self.s_qkv.weight)
        nn.init.xavier_uniform_(self.out_proj.weight)
        _xavier_per_token(self.ns_qkv_weight)

    def forward(self, x: torch.Tensor, n_s: int, q_len: int) -> torch.Tensor:
        """x [B, T, D] (normed) -> out-projected attention of the last q_len
        queries, [B, q_len, D].  On CUDA (no dropout, native impls) all T rows
        are computed and the result is a [B, q_len, D] view of [B, T, D]."""
        B, T, D = x.shape
        qkv = dense.mixed_linear(x, n_s, self.s_qkv.weight, self.ns_qkv_weight)  # [B, T, 3D]
        qkv = qkv.view(B, T, 3, self.n_heads, self.d_head)
        no_drop = not (self.training and self.attn_drop > 0 and self.attention_impl != "fav4")
        if x.is_cuda and self.attention_impl in ("fav4", "fav2", "turbo", "native") and no_drop \
                and _fmha_native_ok(qkv):
            o = pyramid_attention_qkv(qkv, q_len)
            return dense.linear(self.out_proj, o.reshape(B, q_len, D))
        if x.is_cuda and self.attention_impl in ("fav4", "fav2", "turbo", "native") and \
                not (self.training and self.attn_drop > 0 and self.attention_impl != "fav4"):
            o = causal_attention_all_rows(qkv, self.n_heads).reshape(B, T, D)
            return self.out_proj(o)[:, T - q_len:]
        q = qkv[:, T - q_len:, 0]
        k = qkv[:, :, 1]
        v = qkv[:, :, 2]
        impl = {"sdpa": "mask", "native": "native"}.get(self.attention_impl, "auto")
        if not x.is_cuda:
            impl = "mask"
        drop = self.attn_drop if (self.training and self.attention_impl in ("sdpa", "fav2", "turbo")) else 0.0
        out = pyramid_attention(q, k, v, impl=impl, dropout_p=drop)
        return self.out_proj(out.reshape(B, q_len, D))


class MixedFFN(nn.Module):
    def __init__(self, d_model: int, ffn_dim: int, n_ns_tokens: int, dropout: float = 0.0):
        super().__init__()
        self.n_ns = n_ns_tokens
        self.d_model = d_model
        self.s_w1 = nn.Linear(d_model, ffn_dim, bias=False)
        self.s_w2 = nn.Linear(ffn_dim, d_model, bias=False)
        self.ns_w1 = nn.Parameter(torch.empty(n_ns_tokens, ffn_dim, d_model))
        self.ns_w2 = nn.Parameter(torch.empty(n_ns_tokens, d_model, ffn_dim))
        self.dropout = nn.Dropout(dropout)
        nn.init.xavier_uniform_(self.s_w1.weight)
        nn.init.xavier_uniform_(self.s_w2.weight)
        _xavier_per_token(self.ns_w1)
        _xavier_per_token(self.ns_w2)

    def forward(self, x: torch.Tensor, n_s: int) -> torch.Tensor:
        h = dense.mixed_linear(x, n_s, self.s_w1.weight, self.ns_w1, act="gelu")
        h = self.dropout(h)
        return dense.mixed_linear(h, n_s, self.s_w2.weight, self.ns_w2)


class OneTransBlock(nn.Module):
    """Pre-norm block: z = x_tail + Attn(N1(x)); out = z + FFN(N2(z))."""

    def __init__(self, d_model: int, n_heads: int, n_ns_tokens: int, ffn_mult: int = 4,
                 dropout: float = 0.0, attention_impl: str = "sdpa", norm: str = "rmsnorm"):
        super().__init__()
        self.norm1 = make_norm(norm, d_model)
        self.attn = MixedAttention(d_model, n_heads, n_ns_tokens, dropout, attention_impl)
        self.norm2 = make_norm(norm, d_model)
        self.ffn = MixedFFN(d_model, d_model * ffn_mult, n_ns_tokens, dropout)

    def forward(self, x: torch.Tensor, q_len: int, n_s_tokens: int) -> torch.Tensor:
        kv_len = x.shape[1]
        n_ns = kv_len - n_s_tokens
        h, x_tail = norm_with_tail(self.norm1, x, q_len)
        a = self.attn(h, n_s=n_s_tokens, q_len=q_len)
        y, z = add_norm(a, x_tail, self.norm2.weight,
                        getattr(self.norm2, "bias", None), self.norm2.eps, self.norm2.kind)
        fused = dense.mixed_ffn(y, z, q_len - n_ns, self.ffn.s_w1.weight, self.ffn.s_w2.weight,
                                self.ffn.ns_w1, self.ffn.ns_w2) if (self.ffn.dropout.p == 0 or not self.training) else None
        if fused is not None:
            return fused
        f = self.ffn(y, n_s=q_len - n_ns)
        return z + f


class SequentialTokenizer(nn.Module):
    def __init__(self, raw_dim: int, d_model: int, max_len: int = 1024, use_pos_embed: bool = True):
        super().__init__()
        self.proj = nn.Sequential(nn.Linear(raw_dim, d_model), nn.GELU(), nn.Linear(d_model, d_model))
        self.pos_emb = nn.Embedding(max_len, d_model) if use_pos_embed else None

    def forward(self, raw: torch.Tensor) -> torch.Tensor:
        pos = self.pos_emb.weight[: raw.shape[1]] if self.pos_emb is not None else None
        return dense.mlp2(raw, self.proj[0], self.proj[2], addend=pos)


class AutoSplitTokenizer(nn.Module):
    def __init__(self, ns_input_dim: int, d_model: int, n_ns_tokens: int):
        super().__init__()
        out = d_model * n_ns_tokens
        self.proj = nn.Sequential(nn.Linear(ns_input_dim, out), nn.GELU(), nn.Linear(out, out))
        self.n_ns_tokens = n_ns_tokens
        self.d_model = d_model

    def forward(self, ns: torch.Tensor) -> torch.Tensor:
        return dense.mlp2(ns, self.proj[0], self.proj[2]).view(-1, self.n_ns_tokens, self.d_model)


class OneTransModel(BaseModel):
    def __init__(self, config: Config, device: torch.device | None = None, meta_device: bool = False):
        super().__init__()
        self.config = config
        mc, fc, ot = config.model, config.feature, config.model.transformer
        device = torch.device("cpu") if device is None else torch.device(device)
        emb_device = torch.device("meta") if meta_device else device
        self.tasks = list(config.task_names)
        E = mc.embedding_dim
        tc = config.train
        opt = SparseOptimizer(kind=tc.embedding_optimizer, lr=tc.embedding_lr, eps=tc.embedding_eps,
                              weight_decay=tc.weight_decay)
        self.emb = Embeddings(mc.resolved_embedding_tables(), device=emb_device,
                              embedding_init=mc.embedding_init,
                              scalar_feature_names=set(fc.scalar_feature_names), optimizer=opt)
        self.seq_tokenizers = nn.ModuleDict({
            g: SequentialTokenizer(sum(self.emb.feature_dim(f) for f in feats), ot.d_model, max_len=2048,
                                   use_pos_embed=ot.pos_embed)
            for g, feats in fc.sequence_groups.items()
        }).to(device)
        self.dense_projs = nn.ModuleDict()
        ns_raw = sum(self.emb.feature_dim(f) for f in fc.scalar_feature_names)
        for df in fc.dense_features:
            if df.project:
                act = nn.ReLU(inplace=True) if df.activation == "relu" else nn.GELU()
                self.dense_projs[df.name] = nn.Sequential(nn.Linear(df.dim, E, device=device), act)
                ns_raw += E
            else:
                ns_raw += df.dim
        self.ns_raw_dim = ns_raw
        self.ns_tokenizer = AutoSplitTokenizer(ns_raw, ot.d_model, ot.n_ns_tokens).to(device)
        self.blocks = nn.ModuleList([
            OneTransBlock(ot.d_model, ot.n_heads, ot.n_ns_tokens, ot.ffn_mult, ot.dropout,
                          attention_impl=ot.attention_impl, norm=ot.norm)
            for _ in range(ot.n_layers)
        ]).to(device)
        self.final_norm = make_norm(ot.norm, ot.d_model).to(device)
        self.head_proj = nn.Sequential(nn.Linear(ot.n_ns_tokens * ot.d_model, ot.d_model, device=device),
                                       nn.GELU(), nn.Dropout(ot.dropout))
        self.heads = nn.ModuleDict({t: nn.Linear(ot.d_model, 1, device=device) for t in self.tasks})
        self._item_scalar_names = [s.name for s in fc.item_scalar_features]
        self.contrastive_user_proj = nn.Linear(ot.d_model, ot.d_model, device=device)
        self.contrastive_item_proj = nn.Sequential(
            nn.Linear(sum(self.emb.feature_dim(f) for f in self._item_scalar_names) or 1, ot.d_model,
                      device=device), nn.ReLU(inplace=True))

    # ------------------------------------------------------------------
    def get_num_flops_per_sample(self) -> float:
        """Analytic fwd+bwd FLOPs per sample (6x per matmul MAC, 12x attention,
        no causal discount); same accounting as ``onetrans.py:392-474`` with
        per-group history lengths."""
        cfg = self.config
        ot, fc = cfg.model.transformer, cfg.feature
        D, H, n_ns = ot.d_model, ot.n_heads, ot.n_ns_tokens
        dh, F_ = D // H, D * ot.ffn_mult
        L_S = cfg.sequence_length_total()
        sched = pyramid_schedule(L_S, n_ns, ot.n_layers) if ot.use_pyramid else [L_S] * ot.n_layers
        fl = 0
        for g, feats in fc.sequence_groups.items():
            raw = sum(self.emb.feature_dim(f) for f in feats)
            fl += 6 * cfg.data.group_length(g) * (raw * D + D * D)
        for df in fc.dense_features:
            if df.project:
                fl += 6 * df.dim * cfg.model.embedding_dim
        no = n_ns * D
        fl += 6 * (self.ns_raw_dim * no + no * no)
        kv = L_S + n_ns
        for l in range(ot.n_layers):
            q = sched[l] + n_ns
            fl += 6 * (kv - n_ns) * D * 3 * D + 6 * n_ns * 3 * D * D
            fl += 12 * H * dh * q * kv
            fl += 6 * q * D * D
            fl += 6 * (q - n_ns) * D * F_ * 2 + 6 * n_ns * D * F_ * 2
            kv = q
        fl += 6 * n_ns * D * D + 6 * len(self.tasks) * D
        if cfg.train.contrastive_weight > 0:
            fl += 6 * D * D + 6 * len(self._item_scalar_names) * cfg.model.embedding_dim * D
            fl += 6 * D * (cfg.train.batch_size // (cfg.distributed.num_nodes * cfg.distributed.gpus_per_node))
        return float(fl)

    # ------------------------------------------------------------------
    def _compute_dtype(self, batch) -> torch.dtype:
        return torch.bfloat16 if (torch.is_autocast_enabled("cuda") or torch.is_autocast_enabled("cpu")) \
            else torch.float32

    def _lookup(self, batch: dict[str, torch.Tensor]):
        """One fused lookup: every pool's [B, L, G*E] input + the [B, n_scalar*E] NS block."""
        f2k = self.config.feature_to_batch_key()
        fc = self.config.feature
        feats = {}
        for f in fc.all_ec_feature_names():
            k = f2k.get(f, f)
            if k in batch:
                feats[f] = batch[k]
        groups = [list(v) for v in fc.sequence_groups.values()] + [list(fc.scalar_feature_names)]
        outs = self.emb.lookup_groups(feats, groups, dtype=self._compute_dtype(batch))
        return outs[:-1], outs[-1]

    def _backbone(self, batch: dict[str, torch.Tensor]):
        ot = self.config.model.transformer
        pools, scal = self._lookup(batch)
        s_parts = [tok(raw) for tok, raw in zip(self.seq_tokenizers.values(), pools)]
        parts = [scal]
        for df in self.config.feature.dense_features:
            x = batch[df.name]
            parts.append(self._dense_proj(df, x, scal.dtype) if df.name in self.dense_projs else x.to(scal.dtype))
        ns_raw = torch.cat([p.to(scal.dtype) for p in parts], dim=-1)
        ns_tokens = self.ns_tokenizer(ns_raw)
        # one concatenation of every S pool's tokens and the NS tokens
        x = torch.cat(s_parts + [ns_tokens.to(s_parts[0].dtype)], dim=1)
        B = x.shape[0]
        L_NS = ot.n_ns_tokens
        L_S = x.shape[1] - L_NS
        sched = pyramid_schedule(L_S, L_NS, ot.n_layers) if ot.use_pyramid else [L_S] * ot.n_layers
        for l, block in enumerate(self.blocks):
            q_len = sched[l] + L_NS
            x = block(x, q_len=q_len, n_s_tokens=x.shape[1] - L_NS)
        x = self.final_norm(x)
        s_repr = x[:, : x.shape[1] - L_NS].float().mean(dim=1)
        hp = self.head_proj
        h = hp[2](dense.linear(hp[0], x[:, -L_NS:].reshape(B, -1), act="gelu"))
        return h, s_repr, scal

    def _dense_proj(self, df, x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
        """Linear + activation of a projected dense feature (GEMM epilogue on CUDA)."""
        seq = self.dense_projs[df.name]
        act = "relu" if isinstance(seq[1], nn.ReLU) else "gelu"
        return dense.linear(seq[0], x.to(dtype), act=act)

    def forward(self, batch: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
        h, _, _ = self._backbone(batch)
        return {t: head(h).squeeze(-1) for t, head in self.heads.items()}

    def forward_loss(self, batch: dict[str, torch.Tensor], loss_weights: dict[str, float],
                     regression_tasks: list[str]):
        """(total, {task: loss}, {task: logits}) with heads + loss fused."""
        h, _, _ = self._backbone(batch)
        return fused_heads_loss(self.heads, h, batch, loss_weights, regression_tasks)

    # ------------------------------------------------------------------
    @torch.no_grad()
    def score_candidates(self, user_batch: dict[str, torch.Tensor], candidate_batch: dict[str, torch.Tensor],
                         task: str, batch_size: int = 1024) -> torch.Tensor:
        """Scores [C] of one user against C candidates with an S-side K/V cache.

        S tokens sit before the NS tokens and attention is causal, so the S
        stream (hidden states, and the keys / values of every layer) depends
        on the user's history only: it is computed once, for a batch of one,
        following the pyramid. Each candidate then runs only its NS tokens,
        attending to the cached S keys / values plus its own NS keys -- the
        same function as ``forward`` on (user history, candidate), at the cost
        of n_ns tokens per candidate instead of L_S + n_ns
        (``primus_dlrm/evaluation/metrics.py:200-279`` recomputes everything).
        """
        ot = self.config.model.transformer
        n_ns, H = ot.n_ns_tokens, ot.n_heads
        D = ot.d_model
        dh = D // H
        C = next(iter(candidate_batch.values())).shape[0]
        # ---- user side: S tokens through the pyramid, caching per-layer K / V ----
        f2k = self.config.feature_to_batch_key()
        fc = self.config.feature
        seq = {f: user_batch[f2k.get(f, f)] for feats in fc.sequence_groups.values() for f in feats}
        pools = self.emb.lookup_groups(seq, [list(v) for v in fc.sequence_groups.values()],
                                       dtype=self._compute_dtype(user_batch))
        xs = torch.cat([tok(raw) for tok, raw in zip(self.seq_tokenizers.values(), pools)], dim=1)  # [1, L_S, D]
        L_S = xs.shape[1]
        sched = pyramid_schedule(L_S, n_ns, ot.n_layers) if ot.use_pyramid else [L_S] * ot.n_layers
        cache = []
        for l, blk in enumerate(self.blocks):
            at = blk.attn
            h = blk.norm1(xs)
            qkv = (h @ at.s_qkv.weight.t().to(h.dtype)).view(1, -1, 3, H, dh)
            q_s = sched[l]                                   # S queries kept by this layer
            k_s, v_s = qkv[:, :, 1], qkv[:, :, 2]            # [1, n_s, H, dh]
            cache.append((k_s, v_s))
            n_s = xs.shape[1]
            q = qkv[:, n_s - q_s:, 0]
            o = pyramid_attention(q, k_s, v_s, impl="mask").reshape(1, q_s, D)
            z = at.out_proj(o) + xs[:, n_s - q_s:]
            y = blk.norm2(z)
            xs = z + blk.ffn.s_w2(F.gelu(blk.ffn.s_w1(y)))
        # ---- candidate side: NS tokens only ----
        scores = []
        for c0 in range(0, C, batch_size):
            c1 = min(C, c0 + batch_size)
            cb = {k: v[c0:c1] for k, v in candidate_batch.items()}
            nb = c1 - c0
            for k, v in user_batch.items():
                if k not in cb:
                    cb[k] = v.expand(nb, *v.shape[1:])
            ns_raw = self._ns_raw(cb)
            x = self.ns_tokenizer(ns_raw)                    # [nb, n_ns, D]
            for l, blk in enumerate(self.blocks):
                at = blk.attn
                k_s, v_s = cache[l]
                n_s = k_s.shape[1]
                h = blk.norm1(x)
                qkv = torch.einsum("btk,tnk->btn", h, at.ns_qkv_weight.to(h.dtype)).view(nb, n_ns, 3, H, dh)
                q, k_n, v_n = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
                k = torch.cat([k_s.expand(nb, -1, -1, -1).to(k_n.dtype), k_n], dim=1)
                v = torch.cat([v_s.expand(nb, -1, -1, -1).to(v_n.dtype), v_n], dim=1)
                o = pyramid_attention(q, k, v, impl="mask").reshape(nb, n_ns, D)
                z = at.out_proj(o) + x
                y = blk.norm2(z)
                f = torch.einsum("btk,tnk->btn", y, blk.ffn.ns_w1.to(y.dtype))
                f = torch.einsum("btk,tnk->btn", F.gelu(f), blk.ffn.ns_w2.to(y.dtype))
                x = z + f
            x = self.final_norm(x)
            hh = self.head_proj(x.reshape(nb, -1))
            scores.append(self.heads[task](hh).squeeze(-1).float())
        return torch.cat(scores)

    def _ns_raw(self, batch: dict[str, torch.Tensor]) -> torch.Tensor:
        """The NS tokenizer input of a batch: scalar embeddings + dense features."""
        f2k = self.config.feature_to_batch_key()
        fc = self.config.feature
        feats = {f: batch[f2k.get(f, f)] for f in fc.scalar_feature_names if f2k.get(f, f) in batch}
        scal = self.emb.lookup_groups(feats, [list(fc.scalar_feature_names)], dtype=self._compute_dtype(batch))[0]
        parts = [scal]
        for df in fc.dense_features:
            xd = batch[df.name]
            parts.append(self.dense_projs[df.name](xd) if df.name in self.dense_projs else xd.to(scal.dtype))
        return torch.cat([p.to(scal.dtype) for p in parts], dim=-1)

    def forward_with_cross_scores(self, batch: dict[str, torch.Tensor], cross_task: str = ""):
        h, s_repr, scal = self._backbone(batch)
        preds = {t: head(h).squeeze(-1) for t, head in self.heads.items()}
        user = self.contrastive_user_proj(s_repr.to(h.dtype))
        E = self.config.model.embedding_dim
        names = self.config.feature.scalar_feature_names
        cols = []
        for f in self._item_scalar_names:
            i = names.index(f)
            cols.append(scal[:, i * E:(i + 1) * E])
        item = self.contrastive_item_proj(torch.cat(cols, dim=-1))
        return preds, user @ item.t()

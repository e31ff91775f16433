"""Feature-interaction modules (``primus_dlrm/models/interaction.py``).

* ``ConcatMLP``      -- concat + MLP.
* ``DotInteraction`` -- project to a common dim, pairwise dots (upper
  triangle) + the projected features, then the top MLP.
* ``DCNv2``          -- cross layers ``x_{l+1} = x0 * (x_l W + b) + x_l`` with a
  deep MLP in parallel and a combining Linear.  ``low_rank > 0`` factors
  ``W = U V^T`` (rank r), the form the DLRM-DCNv2 benchmark config uses
  (rank 512); ``low_rank = 0`` is the reference's full-rank cross.

On CUDA in bf16 the MLPs and the low-rank cross layers run on the tcgen05
GEMM (``primus_dlrm_b200.ops.mlp``): bias + ReLU in the GEMM epilogues and the
cross layer's ``x0 * (...) + x_l`` fused into its second GEMM.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from primus_dlrm_b200.ops import mlp as native_mlp


def make_mlp(dims: list[int], dropout: float = 0.1, final_activation: bool = True) -> nn.Sequential:
    layers: list[nn.Module] = []
    for i in range(len(dims) - 1):
        layers.append(nn.Linear(dims[i], dims[i + 1]))
        if i < len(dims) - 2 or final_activation:
            layers.append(nn.ReLU(inplace=True))
            if dropout > 0:
                layers.append(nn.Dropout(dropout))
    return nn.Sequential(*layers)


_make_mlp = make_mlp


class InteractionModule(nn.Module):
    output_dim: int

    def forward(self, user_features: list[torch.Tensor], item_features: list[torch.Tensor]) -> torch.Tensor:
        raise NotImplementedError


class ConcatMLP(InteractionModule):
    def __init__(self, input_dim: int, hidden_dims: list[int], dropout: float = 0.1):
        super().__init__()
        self.mlp = make_mlp([input_dim] + hidden_dims, dropout, final_activation=True)
        self.output_dim = hidden_dims[-1]

    def forward(self, user_features, item_features):
        return native_mlp.mlp_chain(self.mlp, torch.cat(list(user_features) + list(item_features), dim=-1))


class DotInteraction(InteractionModule):
    def __init__(self, feature_dims: list[int], top_mlp_dims: list[int], dropout: float = 0.1):
        super().__init__()
        c = max(feature_dims)
        self.projections = nn.ModuleList([nn.Linear(d, c) if d != c else nn.Identity() for d in feature_dims])
        k = len(feature_dims)
        self.top_mlp = make_mlp([k * (k - 1) // 2 + k * c] + top_mlp_dims, dropout, final_activation=True)
        self.output_dim = top_mlp_dims[-1]
        self.common_dim = c
        iu = torch.triu_indices(k, k, offset=1)
        self.register_buffer("_iu", iu, persistent=False)

    def forward(self, user_features, item_features):
        feats = [p(f) for p, f in zip(self.projections, list(user_features) + list(item_features))]
        st = torch.stack(feats, dim=1)
        dots = torch.bmm(st, st.transpose(1, 2))
        pair = dots[:, self._iu[0], self._iu[1]]
        return native_mlp.mlp_chain(self.top_mlp, torch.cat([pair, torch.cat(feats, dim=-1)], dim=-1))


class DCNv2(InteractionModule):
    def __init__(self, input_dim: int, num_cross_layers: int = 3, deep_dims: list[int] | None = None,
                 dropout: float = 0.1, low_rank: int = 0):
        super().__init__()
        self.num_cross_layers = num_cross_layers
        self.low_rank = low_rank
        if low_rank > 0:
            self.cross_u = nn.ParameterList([nn.Parameter(torch.randn(input_dim, low_rank) * 0.01)
                                             for _ in range(num_cross_layers)])
            self.cross_v = nn.ParameterList([nn.Parameter(torch.randn(low_rank, input_dim) * 0.01)
                                             for _ in range(num_cross_layers)])
        else:
            self.cross_weights = nn.ParameterList([nn.Parameter(torch.randn(input_dim, input_dim) * 0.01)
                                                   for _ in range(num_cross_layers)])
        self.cross_biases = nn.ParameterList([nn.Parameter(torch.zeros(input_dim)) for _ in range(num_cross_layers)])
        deep_dims = deep_dims or [input_dim, input_dim]
        self.deep_mlp = make_mlp([input_dim] + deep_dims, dropout, final_activation=True)
        self.combine = nn.Linear(input_dim + deep_dims[-1], deep_dims[-1])
        self.output_dim = deep_dims[-1]

    def cross(self, x0: torch.Tensor) -> torch.Tensor:
        xl = x0
        if self.low_rank > 0 and native_mlp.cross_ok(x0, x0.shape[-1], self.low_rank):
            for i in range(self.num_cross_layers):
                xl = native_mlp.cross_layer(x0, xl, self.cross_u[i], self.cross_v[i], self.cross_biases[i])
            return xl
        for i in range(self.num_cross_layers):
            if self.low_rank > 0:
                proj = (xl @ self.cross_u[i].to(xl.dtype)) @ self.cross_v[i].to(xl.dtype)
            else:
                proj = xl @ self.cross_weights[i].to(xl.dtype)
            xl = x0 * (proj + self.cross_biases[i].to(xl.dtype)) + xl
        return xl

    def forward(self, user_features, item_features):
        x0 = torch.cat(list(user_features) + list(item_features), dim=-1)
        h = torch.cat([self.cross(x0), native_mlp.mlp_chain(self.deep_mlp, x0)], dim=-1)
        return native_mlp.linear(self.combine, h)


def build_interaction(interaction_type: str, user_dims: list[int], item_dims: list[int],
                      top_mlp_dims: list[int], dcn_num_cross_layers: int = 3, dropout: float = 0.1,
                      dcn_low_rank: int = 0) -> InteractionModule:
    total = sum(user_dims) + sum(item_dims)
    if interaction_type == "concat_mlp":
        return ConcatMLP(total, top_mlp_dims, dropout)
    if interaction_type == "dot":
        return DotInteraction(list(user_dims) + list(item_dims), top_mlp_dims, dropout)
    if interaction_type == "dcnv2":
        return DCNv2(total, dcn_num_cross_layers, top_mlp_dims, dropout, low_rank=dcn_low_rank)
    raise ValueError(f"Unknown interaction type: {interaction_type}")

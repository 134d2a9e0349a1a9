"""Graph neural-network layers: GCN, GAT and GraphSAGE (dense adjacency or
adjacency lists; batched over graphs where noted).

  GraphConvLayer       H' = act(D^-1/2 (A + I) D^-1/2 H W + b)   (Kipf & Welling)
  GraphAttentionLayer  e_ij = LeakyReLU(a^T [W h_i || W h_j]) over edges
                       (and self loops), alpha = softmax_j(e_ij), heads
                       concatenated or averaged                  (Velickovic et al.)
  GraphSageLayer       h'_i = act(W_self h_i + W_neigh agg_{j in N(i)} h_j + b),
                       agg = mean or max                         (Hamilton et al.)

Reference parity: scirs2-neural/src/layers/graph_conv.rs:58-900
(GraphActivation, GraphConvLayer with normalised adjacency,
GraphAttentionLayer, GraphSageLayer with Mean / Max aggregators).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

_ACT = {"none": lambda x: x, "relu": F.relu, "sigmoid": torch.sigmoid, "tanh": torch.tanh, "elu": F.elu}


def normalize_adjacency(adj: torch.Tensor) -> torch.Tensor:
    """D^-1/2 (A + I) D^-1/2 for a dense [.., N, N] adjacency."""
    n = adj.shape[-1]
    a = adj + torch.eye(n, device=adj.device, dtype=adj.dtype)
    d = a.sum(-1).clamp_min(1e-12).rsqrt()
    return d.unsqueeze(-1) * a * d.unsqueeze(-2)


class GraphConvLayer(nn.Module):
    def __init__(self, in_features: int, out_features: int, activation: str = "relu", bias: bool = True):
        super().__init__()
        self.lin = nn.Linear(in_features, out_features, bias=False)
        nn.init.xavier_uniform_(self.lin.weight)
        self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None
        self.act = _ACT[activation]

    def forward(self, h: torch.Tensor, adj: torch.Tensor) -> torch.Tensor:
        out = normalize_adjacency(adj) @ self.lin(h)
        if self.bias is not None:
            out = out + self.bias
        return self.act(out)


class GraphAttentionLayer(nn.Module):
    def __init__(self, in_features: int, out_features: int, num_heads: int = 1, concat: bool = True,
                 negative_slope: float = 0.2, activation: str = "elu"):
        super().__init__()
        self.h, self.f, self.concat = num_heads, out_features, concat
        self.W = nn.Linear(in_features, num_heads * out_features, bias=False)
        nn.init.xavier_uniform_(self.W.weight)
        self.a_src = nn.Parameter(torch.empty(num_heads, out_features))
        self.a_dst = nn.Parameter(torch.empty(num_heads, out_features))
        for p in (self.a_src, self.a_dst):
            nn.init.uniform_(p, -1 / math.sqrt(out_features), 1 / math.sqrt(out_features))
        self.slope = negative_slope
        self.act = _ACT[activation]

    def forward(self, h: torch.Tensor, adj: torch.Tensor) -> torch.Tensor:
        n = h.shape[-2]
        z = self.W(h).view(*h.shape[:-1], self.h, self.f)  # [.., N, H, F]
        src = (z * self.a_src).sum(-1)  # [.., N, H]
        dst = (z * self.a_dst).sum(-1)
        e = F.leaky_relu(dst.unsqueeze(-2) + src.unsqueeze(-3), self.slope)  # [.., N(i), N(j), H]
        mask = (adj + torch.eye(n, device=adj.device, dtype=adj.dtype)) > 0
        e = e.masked_fill(~mask.unsqueeze(-1), float("-inf"))
        alpha = torch.softmax(e, dim=-2)
        out = torch.einsum("...ijh,...jhf->...ihf", alpha, z)
        out = out.reshape(*out.shape[:-2], self.h * self.f) if self.concat else out.mean(-2)
        return self.act(out)


class GraphSageLayer(nn.Module):
    def __init__(self, in_features: int, out_features: int, aggregator: str = "mean", activation: str = "relu"):
        super().__init__()
        assert aggregator in ("mean", "max")
        self.w_self = nn.Linear(in_features, out_features)
        self.w_neigh = nn.Linear(in_features, out_features, bias=False)
        self.agg = aggregator
        self.act = _ACT[activation]

    def aggregate(self, h: torch.Tensor, neighbors: list[list[int]]) -> torch.Tensor:
        rows = []
        for nb in neighbors:
            if not nb:
                rows.append(torch.zeros(h.shape[-1], device=h.device, dtype=h.dtype))
            else:
                x = h[nb]
                rows.append(x.mean(0) if self.agg == "mean" else x.max(0).values)
        return torch.stack(rows)

    def forward(self, h: torch.Tensor, neighbors: list[list[int]]) -> torch.Tensor:
        return self.act(self.w_self(h) + self.w_neigh(self.aggregate(h, neighbors)))

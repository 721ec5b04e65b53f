"""Slot-level schedule-search policy (GNN actor-critic).

Module names, shapes and construction order are part of the checkpoint
format and are kept identical to rlccl/models/{gnn_layers,moment_encoder,
slot_policy}.py so that existing checkpoints load strictly:

* ``ECDUGNNLayer``: ``edge_update = [Linear(e + 2n, h), LayerNorm, LeakyReLU(0.1)]``
  over ``[h_edge, h_src, h_dst]``; ``node_update = [Linear(n + 2h, h), LayerNorm,
  LeakyReLU(0.1)]`` over ``[h_node, sum_in, sum_out]``.
* ``MomentEncoder.network = [Linear(g, h), LayerNorm, LeakyReLU, Linear(h, h), LeakyReLU]``.
* ``SlotLevelPolicy``: ``node_encoder``, ``edge_encoder``, ``chunk_encoder``,
  ``layer1``, ``layer2``, ``global_pool``, optional ``moment_encoder`` +
  ``context_fusion`` (only when ``global_moment_feat_dim > 0``), ``actor``
  (input ``4h + cand + h``) and ``critic``.

The in/out aggregation uses ``index_add_`` so it runs on CPU or CUDA.
"""

from __future__ import annotations

import torch
import torch.nn as nn


class ECDUGNNLayer(nn.Module):
    """Edge-centric dual-update message passing layer."""

    def __init__(self, node_dim: int, edge_dim: int, hidden_dim: int):
        super().__init__()
        self.edge_update = nn.Sequential(nn.Linear(edge_dim + 2 * node_dim, hidden_dim),
                                         nn.LayerNorm(hidden_dim), nn.LeakyReLU(0.1))
        self.node_update = nn.Sequential(nn.Linear(node_dim + 2 * hidden_dim, hidden_dim),
                                         nn.LayerNorm(hidden_dim), nn.LeakyReLU(0.1))

    def forward(self, h_nodes, h_edges, edge_src, edge_dst, num_nodes):
        h_e = self.edge_update(torch.cat([h_edges, h_nodes[edge_src], h_nodes[edge_dst]], dim=-1))
        width = h_e.size(1)
        incoming = torch.zeros(num_nodes, width, device=h_nodes.device, dtype=h_e.dtype).index_add_(0, edge_dst, h_e)
        outgoing = torch.zeros(num_nodes, width, device=h_nodes.device, dtype=h_e.dtype).index_add_(0, edge_src, h_e)
        h_v = self.node_update(torch.cat([h_nodes, incoming, outgoing], dim=-1))
        return h_v, h_e


class MomentEncoder(nn.Module):
    """Encodes the global history-only moment vector into the policy context."""

    def __init__(self, global_feat_dim: int, hidden_dim: int):
        super().__init__()
        if global_feat_dim <= 0 or hidden_dim <= 0:
            raise ValueError("global_feat_dim and hidden_dim must be positive")
        self.global_feat_dim = int(global_feat_dim)
        self.network = nn.Sequential(nn.Linear(global_feat_dim, hidden_dim), nn.LayerNorm(hidden_dim),
                                     nn.LeakyReLU(0.1), nn.Linear(hidden_dim, hidden_dim), nn.LeakyReLU(0.1))

    def forward(self, feats: torch.Tensor) -> torch.Tensor:
        if feats.shape[-1] != self.global_feat_dim:
            raise ValueError(f"Expected {self.global_feat_dim} global moment features, got {feats.shape[-1]}")
        return self.network(feats)


class SlotLevelPolicy(nn.Module):
    """Actor scores candidate (chunk, edge) pairs; critic values the slot."""

    def __init__(self, node_feat_dim: int = 5, edge_feat_dim: int = 2, cand_feat_dim: int = 5,
                 chunk_feat_dim: int = 2, hidden_dim: int = 64, global_moment_feat_dim: int = 0):
        super().__init__()
        h = hidden_dim
        self.hidden_dim = h
        self.node_feat_dim = int(node_feat_dim)
        self.edge_feat_dim = int(edge_feat_dim)
        self.cand_feat_dim = int(cand_feat_dim)
        self.chunk_feat_dim = int(chunk_feat_dim)
        self.global_moment_feat_dim = int(global_moment_feat_dim)
        self.node_encoder = nn.Linear(node_feat_dim, h)
        self.edge_encoder = nn.Linear(edge_feat_dim, h)
        self.chunk_encoder = nn.Sequential(nn.Linear(chunk_feat_dim, h), nn.LayerNorm(h), nn.LeakyReLU(0.1))
        self.layer1 = ECDUGNNLayer(h, h, h)
        self.layer2 = ECDUGNNLayer(h, h, h)
        self.global_pool = nn.Sequential(nn.Linear(h, h), nn.LeakyReLU(0.1))
        if self.global_moment_feat_dim > 0:
            self.moment_encoder = MomentEncoder(self.global_moment_feat_dim, h)
            self.context_fusion = nn.Sequential(nn.Linear(2 * h, h), nn.LeakyReLU(0.1))
        self.actor = nn.Sequential(nn.Linear(4 * h + cand_feat_dim + h, h), nn.LeakyReLU(0.1), nn.Linear(h, 1))
        self.critic = nn.Sequential(nn.Linear(h, h), nn.LeakyReLU(0.1), nn.Linear(h, 1))

    def encode_state(self, node_feats, edge_feats, edge_src, edge_dst, chunk_feats, global_moment_feats=None):
        n = node_feats.size(0)
        h_v = self.node_encoder(node_feats)
        h_e = self.edge_encoder(edge_feats)
        h_v, h_e = self.layer1(h_v, h_e, edge_src, edge_dst, n)
        h_v, h_e = self.layer2(h_v, h_e, edge_src, edge_dst, n)
        ctx = self.global_pool(h_v.mean(dim=0))
        if self.global_moment_feat_dim > 0:
            if global_moment_feats is None:
                global_moment_feats = torch.zeros(self.global_moment_feat_dim, dtype=node_feats.dtype,
                                                  device=node_feats.device)
            ctx = self.context_fusion(torch.cat([ctx, self.moment_encoder(global_moment_feats)], dim=-1))
        return h_v, h_e, self.chunk_encoder(chunk_feats), ctx

    def get_value(self, g_ctx):
        return self.critic(g_ctx)

    def get_candidate_logits(self, h_v, h_e, h_c, g_ctx, edge_src, edge_dst, cand_e, cand_c, cand_dynamic_feats):
        g = g_ctx.unsqueeze(0).expand(len(cand_e), -1)
        x = torch.cat([h_e[cand_e], h_v[edge_src[cand_e]], h_v[edge_dst[cand_e]], h_c[cand_c],
                       cand_dynamic_feats, g], dim=-1)
        return self.actor(x).squeeze(-1)


__all__ = ["ECDUGNNLayer", "MomentEncoder", "SlotLevelPolicy"]

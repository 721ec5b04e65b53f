"""Deterministic synthetic inputs and random-init weights of a MoE layer.

Reference-parity recipes (kept identical so that the same seed gives the
same tensors as the reference):
  * tokens of rank r, case i: ``np.random.default_rng(30000 + 101 i + r)``
    standard normal [T, D] float32; token ids ``(i+1)*1e8 + r*1e7 + arange(T)``
    (scripts/run_r3_a0_c0.py:123-152);
  * router: ``torch.Generator().manual_seed(seed)``; W = randn(D, E)*0.1,
    b = randn(E)*0.01 (rlccl/transport/reference_router.py:8-12);
  * experts: W1 = randn(E, in, hid) in^-1/2, b1 = randn(E, hid)*0.01,
    W2 = randn(E, hid, out) hid^-1/2, b2 = randn(E, out)*0.01
    (rlccl/transport/reference_full_moe.py:249-262).
Benchmark recipes: router W ~ N(0, 1/D) so logits are ~N(0, 1) for unit
tokens ("unit_logits"), expert weights ~N(0, 0.02) ("normal002"), drawn on
the target device from a seeded generator.
"""

from __future__ import annotations

from dataclasses import dataclass
import math

import numpy as np
import torch

from .config import CASE_ORDER, MoELayerConfig


@dataclass
class RankInputs:
    tokens: torch.Tensor          # [T, D] compute dtype
    token_ids: torch.Tensor       # [T] int64
    payload_words: np.ndarray     # [T] int64 (reference R3 identity word)
    chunk_bias: torch.Tensor | None   # [C, E] fp32
    block_mask: torch.Tensor | None   # [E] uint8


@dataclass
class LayerWeights:
    router_w: torch.Tensor        # [E, D] compute dtype (kernel layout)
    router_b: torch.Tensor        # [E] fp32
    w1: torch.Tensor              # [E, N1, D]   (N1 = F, or 2F gate|up for SwiGLU)
    b1: torch.Tensor | None       # [E, N1] fp32
    w2: torch.Tensor              # [E, Dout, F]
    b2: torch.Tensor | None       # [E, Dout] fp32
    w_gate: torch.Tensor | None = None   # [E, F, D] SwiGLU gate (oracle layout)
    w_up: torch.Tensor | None = None     # [E, F, D]


def _dtype(cfg: MoELayerConfig) -> torch.dtype:
    return torch.bfloat16 if cfg.dtype == "bf16" else torch.float32


def case_index(cfg: MoELayerConfig) -> int:
    name = cfg.name[3:] if cfg.name.startswith("r4_") else cfg.name
    return CASE_ORDER.index(name) if name in CASE_ORDER else 0


def make_rank_inputs(cfg: MoELayerConfig, rank: int, world: int, device: torch.device,
                     seed: int = 0) -> RankInputs:
    T, D, E = cfg.tokens_per_rank, cfg.hidden, cfg.experts
    if cfg.router_init == "reference":
        ci = case_index(cfg)
        rng = np.random.default_rng(30_000 + ci * 101 + rank + seed)
        tokens = torch.from_numpy(rng.standard_normal((T, D)).astype(np.float32))
        token_ids = (ci + 1) * 100_000_000 + rank * 10_000_000 + np.arange(T, dtype=np.int64)
        first = tokens[:, 0].numpy().view(np.uint32).astype(np.uint64)
        second = tokens[:, 1].numpy().view(np.uint32).astype(np.uint64)
        words = ((first << np.uint64(30)) ^ second ^ token_ids.astype(np.uint64)) & np.uint64((1 << 62) - 1)
        tokens = tokens.to(device=device, dtype=_dtype(cfg))
    else:
        gen = torch.Generator(device=device).manual_seed(1_000_003 * (rank + 1) + seed)
        tokens = torch.randn((T, D), generator=gen, device=device, dtype=torch.float32).to(_dtype(cfg))
        token_ids = (rank + 1) * 10_000_000 + np.arange(T, dtype=np.int64)
        words = token_ids.copy()
    chunk_bias = None
    if cfg.case_bias or cfg.zipf_s > 0 or cfg.hot_phase:
        cb = np.zeros((cfg.chunks, E), dtype=np.float32)
        if cfg.case_bias:
            cb += np.asarray(cfg.case_bias, dtype=np.float32)[None, :E]
        rs = np.random.default_rng(4242 + seed)
        if cfg.zipf_s > 0:
            ranks = rs.permutation(E)
            cb += (-cfg.zipf_s * np.log1p(ranks)).astype(np.float32)[None, :]
        if cfg.hot_phase and cfg.chunks > 1:
            hot = cfg.chunks // 2
            for e in range(E):
                if cfg.owner(e, max(world, 1)) == 0:
                    cb[hot, e] += 2.5
        chunk_bias = torch.from_numpy(cb).to(device)
    block_mask = None
    if cfg.zero_pairs > 0 and world > 1:
        rs = np.random.default_rng(777 + seed)
        pairs = set()
        while len(pairs) < min(cfg.zero_pairs, world * (world - 1)):
            s, d = (int(v) for v in rs.integers(0, world, size=2))
            if s != d:
                pairs.add((s, d))
        bm = np.zeros(E, dtype=np.uint8)
        for s, d in pairs:
            if s == rank:
                for e in range(E):
                    if cfg.owner(e, world) == d:
                        bm[e] = 1
        if bm.sum() >= E - cfg.top_k + 1:  # keep at least top_k routable experts
            bm[:] = 0
        block_mask = torch.from_numpy(bm).to(device)
    return RankInputs(tokens, torch.from_numpy(token_ids).to(device), words.astype(np.int64),
                      chunk_bias, block_mask)


def make_weights(cfg: MoELayerConfig, device: torch.device, seed: int = 0) -> LayerWeights:
    D, E, F, O = cfg.hidden, cfg.experts, cfg.ffn_hidden, cfg.out_dim
    dt = _dtype(cfg)
    if cfg.router_init == "reference":
        g = torch.Generator().manual_seed(cfg.router_seed + seed)
        rw = (torch.randn(D, E, generator=g) * 0.1).float()
        rb = (torch.randn(E, generator=g) * 0.01).float()
    else:
        g = torch.Generator(device=device).manual_seed(cfg.router_seed + seed)
        rw = torch.randn(D, E, generator=g, device=device) * (1.0 if cfg.router_init == "unit_logits" else 0.02) / (
            math.sqrt(D) if cfg.router_init == "unit_logits" else 1.0)
        rb = torch.zeros(E, device=device)
    router_w = rw.t().contiguous().to(device=device, dtype=dt)
    router_b = rb.to(device=device, dtype=torch.float32)
    w_gate = w_up = None
    if cfg.expert_init == "reference":
        g = torch.Generator().manual_seed(cfg.expert_seed + seed)
        a1 = torch.randn(E, D, F, generator=g) * D ** -0.5
        b1 = torch.randn(E, F, generator=g) * 0.01
        a2 = torch.randn(E, F, O, generator=g) * F ** -0.5
        b2 = torch.randn(E, O, generator=g) * 0.01
        w1 = a1.transpose(1, 2).contiguous().to(device=device, dtype=dt)
        w2 = a2.transpose(1, 2).contiguous().to(device=device, dtype=dt)
        b1 = b1.to(device)
        b2 = b2.to(device)
    else:
        g = torch.Generator(device=device).manual_seed(cfg.expert_seed + seed)
        if cfg.activation == "swiglu":
            w_gate = (torch.randn(E, F, D, generator=g, device=device) * 0.02).to(dt)
            w_up = (torch.randn(E, F, D, generator=g, device=device) * 0.02).to(dt)
            w1 = torch.cat([w_gate, w_up], dim=1)  # canonical [gate; up]; kernel interleaves per tile
        else:
            w1 = (torch.randn(E, F, D, generator=g, device=device) * 0.02).to(dt)
        w2 = (torch.randn(E, O, F, generator=g, device=device) * 0.02).to(dt)
        b1 = None
        b2 = None
    return LayerWeights(router_w, router_b, w1, b1, w2, b2, w_gate, w_up)


__all__ = ["LayerWeights", "RankInputs", "case_index", "make_rank_inputs", "make_weights"]

"""MoE layer configuration and named presets.

One dataclass describes a progressive MoE layer instance: tokens per rank,
widths, experts, top-k, router chunking and the reveal policy, expert MLP
shape/activation, compute dtype and expert placement.  Presets cover the
reference's own R3/R4 configurations (scripts/run_r2_f0_integrated.py:59-71,
scripts/run_r4_a0_c0_full_moe.py:50-54) and the five benchmark
configurations of this framework.

Reveal policy: ``partial_shards`` over ``partial_chunks`` progressive chunks
plus a checkpoint at the final chunk — chunks ``0..P-1`` each become one
descriptor as they complete, the remaining chunks are revealed together at
the final trigger and form the last descriptor (P = 3/4 of the chunks by
default, the reference's 75% + checkpoint-8 schedule).
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, field, replace
import json
from typing import Any

ACTIVATIONS = ("relu", "gelu", "silu", "swiglu")
GATE_MODES = {"none": 0, "topk_softmax": 1, "softmax": 2}
MASK_MODES = {"none": 0, "topology_source": 1}
PLACEMENTS = {"modulo": 0, "contiguous": 1}


@dataclass(frozen=True)
class MoELayerConfig:
    name: str
    tokens_per_rank: int
    hidden: int
    experts: int
    top_k: int
    chunk_sizes: tuple[int, ...]
    ffn_hidden: int
    out_dim: int
    activation: str = "relu"
    dtype: str = "fp32"            # fp32 (tf32 tensor-core GEMMs, exact fp32 router) or bf16
    placement: str = "modulo"      # expert e lives on rank e % W (reference) or contiguous blocks
    gate_mode: str = "none"        # combine weights
    mask_mode: str = "none"        # router mask
    partial_chunks: int | None = None
    ctl_per_chunk: int = 6         # control-projection tokens per chunk
    ctl_nodes: int = 4             # nodes of the control topology (Rear4GPU)
    router_init: str = "reference"   # reference: W ~ N(0,1)*0.1, b ~ N(0,1)*0.01 ; normal002: N(0, 0.02)
    expert_init: str = "reference"   # reference: W1 ~ N/sqrt(in) ... ; normal002: N(0, 0.02)
    router_seed: int = 20260805
    expert_seed: int = 20260812
    zipf_s: float = 0.0            # additive Zipf expert bias on the logits (0 = off)
    hot_phase: bool = False        # one chunk routes 80% of tokens to rank 0's experts
    zero_pairs: int = 0            # randomly chosen (src, dst) rank pairs forced to zero tokens
    case_bias: tuple[float, ...] = ()  # reference case families: constant logit bias per expert
    extra: dict = field(default_factory=dict)

    def __post_init__(self) -> None:
        if self.activation not in ACTIVATIONS:
            raise ValueError(f"activation must be one of {ACTIVATIONS}")
        if self.dtype not in ("fp32", "bf16"):
            raise ValueError("dtype must be fp32 or bf16")
        if self.gate_mode not in GATE_MODES or self.mask_mode not in MASK_MODES:
            raise ValueError("bad gate/mask mode")
        if self.placement not in PLACEMENTS:
            raise ValueError("bad placement")
        if sum(self.chunk_sizes) != self.tokens_per_rank:
            raise ValueError("chunk sizes must sum to tokens_per_rank")
        if not 1 <= self.top_k <= min(8, self.experts):
            raise ValueError("top_k must be in 1..min(8, experts)")
        if self.partial_chunks is not None and not 0 <= self.partial_chunks <= self.chunks:
            raise ValueError("partial_chunks outside 0..chunks")

    @property
    def chunks(self) -> int:
        return len(self.chunk_sizes)

    @property
    def progressive_chunks(self) -> int:
        return self.chunks * 3 // 4 if self.partial_chunks is None else self.partial_chunks

    @property
    def chunk_offsets(self) -> tuple[int, ...]:
        out = [0]
        for s in self.chunk_sizes:
            out.append(out[-1] + s)
        return tuple(out)

    @property
    def descriptor_groups(self) -> tuple[tuple[int, ...], ...]:
        p = self.progressive_chunks
        groups = [(c,) for c in range(p)]
        if p < self.chunks:
            groups.append(tuple(range(p, self.chunks)))
        return tuple(groups)

    @property
    def n_desc(self) -> int:
        return len(self.descriptor_groups)

    @property
    def gemm1_n(self) -> int:
        return 2 * self.ffn_hidden if self.activation == "swiglu" else self.ffn_hidden

    def expert_slots(self, world: int) -> int:
        if self.placement == "modulo":
            return -(-self.experts // world)
        if self.experts % world:
            raise ValueError("contiguous placement needs experts divisible by world size")
        return self.experts // world

    def owner(self, expert: int, world: int) -> int:
        return expert % world if self.placement == "modulo" else expert // self.expert_slots(world)

    def slot(self, expert: int, world: int) -> int:
        return expert // world if self.placement == "modulo" else expert % self.expert_slots(world)

    def with_overrides(self, **kw: Any) -> "MoELayerConfig":
        return replace(self, **kw)

    def to_dict(self) -> dict:
        d = asdict(self)
        d["chunk_sizes"] = list(self.chunk_sizes)
        d["case_bias"] = list(self.case_bias)
        return d

    @classmethod
    def from_dict(cls, d: dict) -> "MoELayerConfig":
        d = dict(d)
        d["chunk_sizes"] = tuple(d["chunk_sizes"])
        d["case_bias"] = tuple(d.get("case_bias", ()))
        return cls(**d)

    def to_json(self) -> str:
        return json.dumps(self.to_dict(), sort_keys=True)


def _uniform(chunks: int, size: int) -> tuple[int, ...]:
    return (size,) * chunks


PRESETS: dict[str, MoELayerConfig] = {
    # Reference R4 full MoE: 4096 tokens/rank, D=2048, 4 experts (e % W), top-1,
    # 8 x 512 chunks, expert 2048 -> 32 ReLU -> 16, fp32, topology-source mask.
    "r4_reference": MoELayerConfig(
        name="r4_reference", tokens_per_rank=4096, hidden=2048, experts=4, top_k=1,
        chunk_sizes=_uniform(8, 512), ffn_hidden=32, out_dim=16, activation="relu", dtype="fp32",
        placement="modulo", gate_mode="none", mask_mode="topology_source"),
    # CPU simulated-ranks run: 2 ranks, 4 experts, 1024 tokens/rank, hidden 256,
    # router N(0, 0.02), seeded top-2 over 8 x 128 chunks.
    "cpu_sim_2rank": MoELayerConfig(
        name="cpu_sim_2rank", tokens_per_rank=1024, hidden=256, experts=4, top_k=2,
        chunk_sizes=_uniform(8, 128), ffn_hidden=256, out_dim=256, activation="relu", dtype="fp32",
        placement="contiguous", gate_mode="topk_softmax", router_init="normal002",
        expert_init="normal002"),
    # Full reference MoE layer in fp32 (tf32 tensor cores): 8 experts top-2,
    # 1024 -> 4096 GELU -> 1024, softmax-gated combine.
    "full_tf32": MoELayerConfig(
        name="full_tf32", tokens_per_rank=4096, hidden=1024, experts=8, top_k=2,
        chunk_sizes=_uniform(8, 512), ffn_hidden=4096, out_dim=1024, activation="gelu", dtype="fp32",
        placement="contiguous", gate_mode="topk_softmax", router_init="unit_logits",
        expert_init="normal002"),
    # Skewed-traffic stress, bf16: 16 experts (2 per rank at 8 GPUs), SwiGLU
    # 2048 -> 8192 -> 2048, top-2, 16 chunks, Zipf bias + hot phase + zero pairs.
    "skewed_bf16": MoELayerConfig(
        name="skewed_bf16", tokens_per_rank=8192, hidden=2048, experts=16, top_k=2,
        chunk_sizes=_uniform(16, 512), ffn_hidden=8192, out_dim=2048, activation="swiglu",
        dtype="bf16", placement="contiguous", gate_mode="topk_softmax", router_init="unit_logits",
        expert_init="normal002", zipf_s=1.2, hot_phase=True, zero_pairs=2),
    # Mixtral-8x7B-shaped: 16384 tokens/rank, 4096, SwiGLU 4096 -> 14336 -> 4096,
    # 8 experts top-2, 32 x 512 chunks, bf16.
    "mixtral_8x7b": MoELayerConfig(
        name="mixtral_8x7b", tokens_per_rank=16384, hidden=4096, experts=8, top_k=2,
        chunk_sizes=_uniform(32, 512), ffn_hidden=14336, out_dim=4096, activation="swiglu",
        dtype="bf16", placement="contiguous", gate_mode="topk_softmax", router_init="unit_logits",
        expert_init="normal002"),
    # DeepSeek-V2-Lite-shaped: 64 routed experts top-6, 2048, SwiGLU
    # 2048 -> 1408 -> 2048, 8192 tokens/rank, 16 chunks, bf16.
    "deepseek_v2_lite": MoELayerConfig(
        name="deepseek_v2_lite", tokens_per_rank=8192, hidden=2048, experts=64, top_k=6,
        chunk_sizes=_uniform(16, 512), ffn_hidden=1408, out_dim=2048, activation="swiglu",
        dtype="bf16", placement="contiguous", gate_mode="softmax", router_init="unit_logits",
        expert_init="normal002"),
}

# The reference R3/R4 correctness case families (scripts/run_r3_a0_c0.py:68-94).
CASE_ORDER = ("balanced", "skewed", "all_to_one_like", "zero_sized_pair", "empty_shard",
              "single_token_shard", "multiple_progressive_shards")
CASE_SPECS = {
    "balanced": {"chunk_sizes": _uniform(8, 512), "bias": (0.0, 0.0, 0.0, 0.0)},
    "skewed": {"chunk_sizes": _uniform(8, 512), "bias": (100.0, 0.0, 0.0, 0.0)},
    "all_to_one_like": {"chunk_sizes": _uniform(8, 512), "bias": (100.0, 0.0, 50.0, 0.0)},
    "zero_sized_pair": {"chunk_sizes": _uniform(8, 512), "bias": (0.0, 100.0, 0.0, 50.0)},
    "empty_shard": {"chunk_sizes": (512, 512, 0, 512, 512, 512, 512, 1024), "bias": (0.0,) * 4},
    "single_token_shard": {"chunk_sizes": (512, 1, 512, 512, 512, 512, 512, 1023), "bias": (0.0,) * 4},
    "multiple_progressive_shards": {"chunk_sizes": (128, 256, 384, 512, 640, 768, 512, 896),
                                    "bias": (0.0,) * 4},
}


def preset(name: str, **overrides: Any) -> MoELayerConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown MoE preset {name!r}; have {sorted(PRESETS)}")
    cfg = PRESETS[name]
    return cfg.with_overrides(**overrides) if overrides else cfg


def r4_case(case: str) -> MoELayerConfig:
    spec = CASE_SPECS[case]
    return PRESETS["r4_reference"].with_overrides(
        name=f"r4_{case}", chunk_sizes=tuple(spec["chunk_sizes"]), case_bias=tuple(spec["bias"]))


def load_config(path: str, **overrides: Any) -> MoELayerConfig:
    """Load a config from JSON or YAML (a ``preset`` key selects a base preset)."""
    with open(path, "r", encoding="utf-8") as f:
        text = f.read()
    if path.endswith((".yaml", ".yml")):
        import yaml

        data = yaml.safe_load(text)
    else:
        data = json.loads(text)
    base = data.pop("preset", None)
    if base is not None:
        if "chunk_sizes" in data:
            data["chunk_sizes"] = tuple(data["chunk_sizes"])
        cfg = preset(base, **data)
    else:
        cfg = MoELayerConfig.from_dict(data)
    return cfg.with_overrides(**overrides) if overrides else cfg


__all__ = ["CASE_ORDER", "CASE_SPECS", "MoELayerConfig", "PRESETS", "load_config", "preset", "r4_case"]

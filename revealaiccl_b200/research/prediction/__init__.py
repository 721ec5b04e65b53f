"""History-only traffic-summary prediction study (rlccl/prediction/*):
preregistered sequences and splits, leakage-safe examples, point methods
(long-term mean, previous value, EWMA, moment ridge, recent-history MLP,
causal TCN), pooled residual calibration, sequence-level statistics and the
seven-condition H1 gate, plus an experiment runner with artifact bundles."""

from .data import FORMAL_BASE_SEEDS, FORMAL_FAMILIES, SequenceSpec, build_formal_sequence_specs
from .models import METHOD_NAMES

__all__ = ["FORMAL_BASE_SEEDS", "FORMAL_FAMILIES", "METHOD_NAMES", "SequenceSpec", "build_formal_sequence_specs"]

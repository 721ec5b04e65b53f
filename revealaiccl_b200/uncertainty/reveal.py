"""Deterministic, monotone partial-demand reveal (rlccl/uncertainty/reveal.py:14-174).

Modes: ``random_entries``, ``source_totals_first``,
``source_destination_totals_first``, ``partial_shards`` and
``time_based_arrival``.  Ratios start at 0, end at 1 and strictly increase.
The generator draws, in this order, an entry permutation, per-entry arrival
times in (0, 1) and a token permutation from ``np.random.default_rng(seed)``
so the same seed reveals the same tokens in the same order as the reference.

* ``partial_shards``: stage ratio r reveals the first floor(r * tokens) tokens
  of the token permutation; a (src, dst) entry is known once all of its
  tokens are revealed (or r == 1).
* entry modes: reveal whole (src, dst) entries — the first floor(r * entries)
  of the entry permutation, or those whose arrival time is <= r.
"""

from __future__ import annotations

import math
from typing import Iterator, Sequence

import numpy as np

from .observation import PartialObservationState, RevealedDemandToken
from .problem import UncertainProblemInstance

MODES = frozenset({"random_entries", "source_totals_first", "source_destination_totals_first",
                   "partial_shards", "time_based_arrival"})


class DemandRevealProcess:
    def __init__(self, *, problem: UncertainProblemInstance, mode: str, ratios: Sequence[float],
                 seed: int) -> None:
        if not isinstance(problem, UncertainProblemInstance):
            raise TypeError("problem must be UncertainProblemInstance")
        if mode not in MODES:
            raise ValueError(f"Unsupported reveal mode: {mode}")
        r = tuple(float(v) for v in ratios)
        if not r or r[0] != 0.0 or r[-1] != 1.0:
            raise ValueError("Reveal ratios must start at 0 and end at 1")
        if any(not math.isfinite(v) or v < 0 or v > 1 for v in r):
            raise ValueError("Reveal ratios must be finite values in [0, 1]")
        if any(a >= b for a, b in zip(r, r[1:])):
            raise ValueError("Reveal ratios must be strictly increasing")
        self._problem = problem
        self._mode = str(mode)
        self._ratios = r
        self._seed = int(seed)
        rng = np.random.default_rng(self._seed)
        n = problem._node_count
        entries = np.asarray([(s, d) for s in range(n) for d in range(n) if s != d],
                             dtype=np.int64).reshape(-1, 2)
        self._entry_order = entries[rng.permutation(len(entries))]
        self._arrival = rng.uniform(np.nextafter(0.0, 1.0), 1.0, size=len(entries))
        self._token_order = rng.permutation(problem._token_count)

    @property
    def ratios(self) -> tuple[float, ...]:
        return self._ratios

    @property
    def mode(self) -> str:
        return self._mode

    def __iter__(self) -> Iterator[PartialObservationState]:
        for stage, ratio in enumerate(self._ratios):
            yield self._build(stage, ratio)

    def observation_for_slot(self, slot: int) -> PartialObservationState:
        """Stage r arrives right before slot r; later slots see the final stage
        rebuilt from the current possession state."""
        if isinstance(slot, (bool, np.bool_)) or not isinstance(slot, (int, np.integer)):
            raise TypeError("slot must be a nonnegative integer")
        if int(slot) < 0:
            raise ValueError("slot must be nonnegative")
        stage = min(int(slot), len(self._ratios) - 1)
        return self._build(stage, self._ratios[stage])

    def observation_for_stage(self, stage: int) -> PartialObservationState:
        if isinstance(stage, (bool, np.bool_)) or not isinstance(stage, (int, np.integer)):
            raise TypeError("stage must be an integer")
        if int(stage) < 0 or int(stage) >= len(self._ratios):
            raise ValueError("stage is outside the reveal schedule")
        return self._build(int(stage), self._ratios[int(stage)])

    def full_observation(self) -> PartialObservationState:
        last = len(self._ratios) - 1
        return self._build(last, self._ratios[last])

    def _revealed(self, ratio: float) -> tuple[np.ndarray, list[int]]:
        world = self._problem
        n = world._node_count
        entry_mask = np.eye(n, dtype=bool)
        indices: list[int] = []
        if self._mode == "partial_shards":
            count = world._token_count if ratio == 1.0 else int(math.floor(ratio * world._token_count))
            indices = [int(v) for v in self._token_order[:count]]
            per_pair: dict[tuple[int, int], int] = {}
            for t in indices:
                s, d, _ = world._atomic[t]
                per_pair[(s, d)] = per_pair.get((s, d), 0) + 1
            for s in range(n):
                for d in range(n):
                    if s == d:
                        continue
                    total = len(world._indices_for_pair(s, d))
                    if ratio == 1.0 or (total > 0 and per_pair.get((s, d), 0) == total):
                        entry_mask[s, d] = True
        else:
            if self._mode == "time_based_arrival":
                selected = self._entry_order if ratio == 1.0 else self._entry_order[self._arrival <= ratio]
            else:
                denom = len(self._entry_order)
                count = denom if ratio == 1.0 else int(math.floor(ratio * denom))
                selected = self._entry_order[:count]
            for s, d in selected:
                entry_mask[int(s), int(d)] = True
                indices.extend(world._indices_for_pair(int(s), int(d)))
        return entry_mask, indices

    def _build(self, stage: int, ratio: float) -> PartialObservationState:
        world = self._problem
        entry_mask, indices = self._revealed(ratio)
        observed = np.zeros_like(world._truth)
        if self._mode == "partial_shards":
            for t in indices:
                s, d, _ = world._atomic[t]
                observed[s, d] += 1
        else:
            observed[entry_mask] = world._truth[entry_mask]
        tokens = []
        for t in indices:
            s, d, holders = world._token_record(t)
            tokens.append(RevealedDemandToken(world._issue_token_id(t, reveal_seed=self._seed), s, d, holders))
        src_tot = dst_tot = None
        if self._mode in ("source_totals_first", "source_destination_totals_first"):
            src_tot = world._truth.sum(axis=1)
        if self._mode == "source_destination_totals_first":
            dst_tot = world._truth.sum(axis=0)
        return PartialObservationState(
            sequence_id=world.sequence_id, sequence_step=world.sequence_step, family=world.family,
            mode=self._mode, stage=int(stage), ratio=float(ratio), entry_mask=entry_mask,
            observed_matrix=observed, unknown_mask=~entry_mask, revealed_tokens=tuple(tokens),
            source_totals=src_tot, destination_totals=dst_tot, topology=world.public_topology,
            state_version=world._state_version,
        )


__all__ = ["DemandRevealProcess", "MODES"]

"""Scheduling: the uncompiled reference planner (oracle) and the compiled,
incremental, fail-closed fast path with its C++ core (layer L4)."""

from .compiled import (BoundBatch, CompiledEventDrivenRuntime, CompiledPlan, DynamicGuard, FastBinder,
                       GuardDecision, IncrementalState, RouteTemplate, RuntimeStep, StateDigest,
                       StaticPlanCompiler, StaticProof, structural_signature)
from .recourse import bind_action
from .robust_prefix import (CandidateAction, RobustPrefixConfig, RobustPrefixPlanner, atomic_units,
                            build_scheduling_view, canonical_shortest_path, enumerate_candidates,
                            pack_candidate_batch)

__all__ = [
    "BoundBatch", "CandidateAction", "CompiledEventDrivenRuntime", "CompiledPlan", "DynamicGuard",
    "FastBinder", "GuardDecision", "IncrementalState", "RobustPrefixConfig", "RobustPrefixPlanner",
    "RouteTemplate", "RuntimeStep", "StateDigest", "StaticPlanCompiler", "StaticProof",
    "atomic_units", "bind_action", "build_scheduling_view", "canonical_shortest_path",
    "enumerate_candidates", "pack_candidate_batch", "structural_signature",
]

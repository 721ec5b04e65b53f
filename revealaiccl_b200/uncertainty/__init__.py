"""Reveal-aware truth / observation / proposal / trusted-checker semantics (layer L3).

This is the oracle every compiled scheduler path and every device kernel is
checked against: evaluator-private truth worlds, deterministic reveal
processes, the planner-facing observation, proposals and the trusted
``commit_proposal`` checker, the baseline policies and the paired evaluator.
"""

from . import baselines, evaluation, execution, metrics, observation, problem, reveal, scenarios
from .baselines import (FullInformationOracle, LongTermMeanBaseline, PartialCurrentOnlyBaseline,
                        PreviousValueBaseline, WaitUntilKnownBaseline)
from .evaluation import EvaluationManifest, PairedEvaluationRunner, RecourseMetrics
from .execution import CommitResult, Proposal, TransferAction, commit_proposal, validate_legacy_schedule_matrix
from .observation import (PartialObservationState, PublicTopologyView, RevealedDemandToken,
                          SanitizedHistoryView, TruthTokenId)
from .problem import UncertainProblemInstance
from .reveal import DemandRevealProcess
from .scenarios import ScenarioDemandToken, ScenarioSet, ScenarioTokenId

__all__ = [
    "CommitResult", "DemandRevealProcess", "EvaluationManifest", "FullInformationOracle",
    "LongTermMeanBaseline", "PairedEvaluationRunner", "PartialCurrentOnlyBaseline",
    "PartialObservationState", "PreviousValueBaseline", "Proposal", "PublicTopologyView",
    "RecourseMetrics", "RevealedDemandToken", "SanitizedHistoryView", "ScenarioDemandToken",
    "ScenarioSet", "ScenarioTokenId", "TransferAction", "TruthTokenId", "UncertainProblemInstance",
    "WaitUntilKnownBaseline", "commit_proposal", "validate_legacy_schedule_matrix",
]

"""Raw reveal-aware recourse metric rows (rlccl/uncertainty/metrics.py)."""

from .evaluation import RecourseMetrics

__all__ = ["RecourseMetrics"]

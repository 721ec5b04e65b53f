"""Neural models: the slot-level schedule policy (GNN actor-critic) and its layers."""

from .policy import ECDUGNNLayer, MomentEncoder, SlotLevelPolicy

__all__ = ["ECDUGNNLayer", "MomentEncoder", "SlotLevelPolicy"]

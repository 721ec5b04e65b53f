"""Host runtime pieces around the device pipeline (completion bridge)."""

from .event_bridge import CompletionBridge, HostFlag

__all__ = ["CompletionBridge", "HostFlag"]

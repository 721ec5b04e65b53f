"""Topology formats, loaders and problem records (layers L0/L1)."""

from .info import ProblemInstance, TopologyInfo, compute_received_chunks, hop_distances, normalize_capacities
from .loader import (
    BUNDLED, available_topologies, build_multi_server_topology, build_nvswitch_topology,
    build_ring_topology, ensure_bundled, load_rear4_topology, load_topology_from_json,
    load_topology_info, parse_topology, topology_path, write_topology,
)

__all__ = [
    "BUNDLED", "ProblemInstance", "TopologyInfo", "available_topologies",
    "build_multi_server_topology", "build_nvswitch_topology", "build_ring_topology",
    "compute_received_chunks", "ensure_bundled", "hop_distances", "load_rear4_topology",
    "load_topology_from_json", "load_topology_info", "normalize_capacities", "parse_topology",
    "topology_path", "write_topology",
]

"""Topology JSON loading and B200 topology construction.

File format (same schema as the reference's
``Data/<name>/Topology/pipeline_topology_no_switch.json``)::

    {"directed": true, "multigraph": true, "graph": {},
     "nodes": [{"id", "role", "physical", "gpu_index"?}, ...],
     "links": [{"source", "target", "capacity_value", "capacity_unit", "type"}, ...],
     "bandwidth_groups": {name: {"max_bandwidth", "bandwidth_unit", "description",
                                 "edges": [{"source", "target"}, ...]}}}

Node ids map to indices in file order; edge index = link order; a
bandwidth group becomes one shared constraint over the edges it names that
exist.  ``load_topology_info`` divides capacities and group limits by the
minimum link capacity, as rlccl/envs/evaluator.py:359-388 does.

``build_nvswitch_topology`` writes the single-NVSwitch-domain topology of an
n-GPU B200 node (every GPU reaches every peer directly; per-GPU egress and
ingress shares are bandwidth groups), which is what the MoE control plane's
scheduler projection runs on.
"""

from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path
from typing import Any

import numpy as np

from .info import TopologyInfo, normalize_capacities

TOPOLOGY_FILE = "pipeline_topology_no_switch.json"
_DATA_DIR = Path(__file__).resolve().parent / "data"


def data_dir() -> Path:
    """Directory holding the bundled topology folders (``<name>/Topology/*.json``);
    ``RAICCL_TOPOLOGY_DIR`` overrides it."""
    override = os.environ.get("RAICCL_TOPOLOGY_DIR")
    return Path(override) if override else _DATA_DIR


def parse_topology(data: dict) -> tuple[int, int, np.ndarray, np.ndarray, list]:
    nodes = data.get("nodes", [])
    links = data.get("links", [])
    index = {node["id"]: i for i, node in enumerate(nodes)}
    edges = np.asarray(
        [[index[link["source"]], index[link["target"]]] for link in links], dtype=np.int64
    ).reshape(-1, 2)
    capacities = np.asarray([float(link.get("capacity_value", 1.0)) for link in links],
                            dtype=np.float64)
    edge_index: dict[tuple[int, int], int] = {}
    for i, (u, v) in enumerate(edges.tolist()):
        edge_index[(u, v)] = i  # a repeated (u, v) link: groups name its last occurrence
    shared: list[tuple[list[int], float]] = []
    for group in data.get("bandwidth_groups", {}).values():
        if not isinstance(group, dict) or "edges" not in group or "max_bandwidth" not in group:
            continue
        members = []
        for e in group["edges"]:
            key = (index[e["source"]], index[e["target"]])
            if key in edge_index:
                members.append(edge_index[key])
        if members:
            shared.append((members, float(group["max_bandwidth"])))
    return len(nodes), len(edges), edges, capacities, shared


def load_topology_from_json(json_path: str | os.PathLike) -> tuple[int, int, np.ndarray, np.ndarray, list]:
    with open(json_path, "r", encoding="utf-8") as f:
        return parse_topology(json.load(f))


def topology_path(name: str, root: str | os.PathLike | None = None) -> Path:
    base = Path(root) if root is not None else data_dir()
    return base / name / "Topology" / TOPOLOGY_FILE


def load_topology_info(name: str, root: str | os.PathLike | None = None,
                       cache: bool = False) -> TopologyInfo:
    path = topology_path(name, root)
    if not path.exists():
        raise FileNotFoundError(f"Topology file not found: {path}")
    V, E, edges, caps, shared = load_topology_from_json(path)
    caps, shared = normalize_capacities(caps, shared)
    return TopologyInfo(V, E, edges, caps, shared,
                        cache_dir=str(path.parent) if cache else None, name=name)


def node_roles(name: str, root: str | os.PathLike | None = None) -> list[str]:
    """The ``role`` of every node of a topology file, in node order ("gpu",
    "switch", "nic", ...); nodes without one count as GPUs."""
    path = topology_path(name, root)
    with open(path, "r", encoding="utf-8") as f:
        data = json.load(f)
    return [str(n.get("role", "gpu")).lower() for n in data.get("nodes", [])]


def file_sha256(path: str | os.PathLike) -> str:
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def available_topologies(root: str | os.PathLike | None = None) -> list[str]:
    base = Path(root) if root is not None else data_dir()
    if not base.exists():
        return []
    return sorted(p.name for p in base.iterdir() if (p / "Topology" / TOPOLOGY_FILE).exists())


# ---------------------------------------------------------------------------
# Builders (produce the JSON schema above)
# ---------------------------------------------------------------------------

def _node(i: int, role: str, physical: str, gpu_index: int | None = None) -> dict:
    n: dict[str, Any] = {"role": role, "physical": physical, "id": i}
    if gpu_index is not None:
        n["gpu_index"] = gpu_index
    return n


def build_nvswitch_topology(num_gpus: int, link_gbps: float = 900.0) -> dict:
    """Single NVSwitch domain: a directed link between every GPU pair and one
    egress + one ingress bandwidth group per GPU (each capped at the per-GPU
    NVLink bandwidth)."""
    if num_gpus < 2:
        raise ValueError("an NVSwitch topology needs at least two GPUs")
    nodes = [_node(i, "gpu", f"GPU{i}", i) for i in range(num_gpus)]
    links = [
        {"source": u, "target": v, "capacity_value": float(link_gbps), "capacity_unit": "GBps",
         "type": "nvlink"}
        for u in range(num_gpus) for v in range(num_gpus) if u != v
    ]
    groups: dict[str, Any] = {}
    for g in range(num_gpus):
        groups[f"nvswitch_gpu{g}_egress"] = {
            "max_bandwidth": float(link_gbps), "bandwidth_unit": "GBps",
            "description": f"Per-GPU NVSwitch egress share (node_id={g})",
            "edges": [{"source": g, "target": v} for v in range(num_gpus) if v != g],
        }
    for g in range(num_gpus):
        groups[f"nvswitch_gpu{g}_ingress"] = {
            "max_bandwidth": float(link_gbps), "bandwidth_unit": "GBps",
            "description": f"Per-GPU NVSwitch ingress share (node_id={g})",
            "edges": [{"source": u, "target": g} for u in range(num_gpus) if u != g],
        }
    return {"directed": True, "multigraph": True, "graph": {}, "nodes": nodes, "links": links,
            "bandwidth_groups": groups}


def build_multi_server_topology(servers: int, gpus_per_server: int, nvlink_gbps: float = 900.0,
                                nic_gbps: float = 50.0, shared_nic: bool = False) -> dict:
    """GPUs fully connected inside each server (NVSwitch), one NIC node per
    server (or per GPU when ``shared_nic`` is False) joined by a network
    switch node.  Cross-server traffic crosses GPU->NIC->switch->NIC->GPU."""
    nodes: list[dict] = []
    links: list[dict] = []
    groups: dict[str, Any] = {}

    def link(u, v, cap, kind):
        links.append({"source": u, "target": v, "capacity_value": float(cap),
                      "capacity_unit": "GBps", "type": kind})

    gpu_ids: list[list[int]] = []
    nid = 0
    for s in range(servers):
        row = []
        for g in range(gpus_per_server):
            nodes.append(_node(nid, "gpu", f"S{s}GPU{g}", s * gpus_per_server + g))
            row.append(nid)
            nid += 1
        gpu_ids.append(row)
    nic_ids: list[list[int]] = []
    for s in range(servers):
        count = 1 if shared_nic else gpus_per_server
        row = []
        for i in range(count):
            nodes.append(_node(nid, "nic", f"S{s}NIC{i}"))
            row.append(nid)
            nid += 1
        nic_ids.append(row)
    switch = nid
    nodes.append(_node(switch, "switch", "NetSwitch"))
    for s in range(servers):
        for a in gpu_ids[s]:
            for b in gpu_ids[s]:
                if a != b:
                    link(a, b, nvlink_gbps, "nvlink")
        for i, g in enumerate(gpu_ids[s]):
            nic = nic_ids[s][0 if shared_nic else i]
            link(g, nic, nic_gbps, "pcie")
            link(nic, g, nic_gbps, "pcie")
        for nic in nic_ids[s]:
            link(nic, switch, nic_gbps, "network")
            link(switch, nic, nic_gbps, "network")
        if shared_nic:
            nic = nic_ids[s][0]
            groups[f"server{s}_nic_egress"] = {
                "max_bandwidth": float(nic_gbps), "bandwidth_unit": "GBps",
                "description": f"Shared NIC uplink of server {s}",
                "edges": [{"source": g, "target": nic} for g in gpu_ids[s]],
            }
    return {"directed": True, "multigraph": True, "graph": {}, "nodes": nodes, "links": links,
            "bandwidth_groups": groups}


def build_ring_topology(num_gpus: int, link_gbps: float = 100.0) -> dict:
    nodes = [_node(i, "gpu", f"GPU{i}", i) for i in range(num_gpus)]
    links = []
    for i in range(num_gpus):
        for j in ((i + 1) % num_gpus, (i - 1) % num_gpus):
            links.append({"source": i, "target": j, "capacity_value": float(link_gbps),
                          "capacity_unit": "GBps", "type": "nvlink"})
    return {"directed": True, "multigraph": True, "graph": {}, "nodes": nodes, "links": links,
            "bandwidth_groups": {}}


def write_topology(data: dict, name: str, root: str | os.PathLike | None = None) -> Path:
    path = topology_path(name, root)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps(data, indent=2) + "\n", encoding="utf-8")
    return path


BUNDLED = {
    "Rear4GPU": lambda: build_nvswitch_topology(4, 200.0),
    "B200_NVSwitch_2GPU": lambda: build_nvswitch_topology(2, 900.0),
    "B200_NVSwitch_4GPU": lambda: build_nvswitch_topology(4, 900.0),
    "B200_NVSwitch_8GPU": lambda: build_nvswitch_topology(8, 900.0),
    "B200_2Server_16GPU": lambda: build_multi_server_topology(2, 8, 900.0, 50.0, shared_nic=False),
    "B200_2Server_16GPU_SameNIC": lambda: build_multi_server_topology(2, 8, 900.0, 50.0, shared_nic=True),
    "Ring6GPU": lambda: build_ring_topology(6, 100.0),
}


def ensure_bundled(root: str | os.PathLike | None = None) -> list[str]:
    """Write every bundled topology that is missing; returns their names."""
    for name, make in BUNDLED.items():
        if not topology_path(name, root).exists():
            write_topology(make(), name, root)
    return sorted(BUNDLED)


def load_rear4_topology() -> tuple[TopologyInfo, str]:
    """The 4-node NVSwitch topology the MoE control-plane projection schedules on,
    plus the sha256 of its file (rlccl/uncertainty/ambiguity_experiment.py:1502)."""
    path = topology_path("Rear4GPU")
    if not path.exists():
        write_topology(BUNDLED["Rear4GPU"](), "Rear4GPU")
    return load_topology_info("Rear4GPU"), file_sha256(path)

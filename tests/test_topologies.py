"""Topology files: all eleven reference topology folders load, and (when the
reference tree is installed under baseline/_ref) parse and normalise exactly
as its evaluator does (rlccl/envs/evaluator.py:36-81, 359-388)."""

import importlib.util
from pathlib import Path

import numpy as np
import pytest

from revealaiccl_b200.topology.loader import (available_topologies, load_topology_from_json, load_topology_info,
                                             topology_path)

REFERENCE_TOPOLOGIES = (
    "Heterogeneous_12GPU", "Heterogeneous_16GPU_3Server", "Heterogeneous_32GPU_4Server",
    "Heterogeneous_32GPU_4Server_PerGPU_NIC", "Heterogeneous_32GPU_4Server_SameNICConnect",
    "Heterogeneous_64GPU_8Server", "Heterogeneous_64GPU_8Server_SameNICConnect", "Heterogeneous_6GPU_Ring",
    "Rear4GPU", "Rear8GPU_NoSwitch_Test", "Rear8GPU_NoSwitch_Test_SameNICConnect",
)
REF_ROOT = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def test_all_reference_topologies_bundled_and_loadable():
    names = set(available_topologies())
    assert set(REFERENCE_TOPOLOGIES) <= names
    for name in REFERENCE_TOPOLOGIES:
        info = load_topology_info(name)
        assert info.V > 0 and info.E > 0 and len(info.capacities) == info.E
        assert float(np.min(info.capacities)) == pytest.approx(1.0)
        for members, limit in info.shared_constraints:
            assert all(0 <= e < info.E for e in members) and limit > 0


def _reference_loader():
    path = REF_ROOT / "rlccl" / "envs" / "evaluator.py"
    if not path.exists():
        return None
    import sys

    sys.path.insert(0, str(REF_ROOT))
    try:
        spec = importlib.util.spec_from_file_location("_ref_evaluator", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    except Exception:
        return None
    return mod


@pytest.mark.parametrize("name", REFERENCE_TOPOLOGIES)
def test_parse_and_normalise_match_reference(name):
    ref = _reference_loader()
    if ref is None:
        pytest.skip("reference tree not installed under baseline/_ref")
    p = topology_path(name)
    V, E, edges, caps, shared = load_topology_from_json(p)
    rV, rE, redges, rcaps, rshared = ref.load_topology_from_json(str(p))
    assert (V, E) == (rV, rE)
    assert np.array_equal(edges, np.asarray(redges))
    assert np.allclose(caps, np.asarray(rcaps, dtype=np.float64))
    assert [(list(m), float(l)) for m, l in shared] == [(list(m), float(l)) for m, l in rshared]
    info = load_topology_info(name)
    m = float(np.min(np.asarray(rcaps, dtype=np.float64)))
    assert np.allclose(info.capacities, np.asarray(rcaps, dtype=np.float64) / m)
    assert [(list(a), pytest.approx(b)) for a, b in info.shared_constraints] == \
        [(list(a), float(b) / m) for a, b in rshared]

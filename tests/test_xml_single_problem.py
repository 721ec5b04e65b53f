"""MSCCL XML lowering (switch back-tracing, collective layouts, threadblock
and dependency lowering, instances, receive-copy-send fusion, simulation
check) and the single-problem CLI."""

import json
import xml.etree.ElementTree as ET

import numpy as np
import pytest
import torch

from revealaiccl_b200.rl import xml_export as X


def _sched(T, C, E, moves):
    out = [np.zeros((C, E), dtype=np.int64) for _ in range(T)]
    for t, c, e in moves:
        out[t][c, e] = 1
    return out


def _ring_allgather(V=4, cf=1):
    """Chunk i starts on GPU i // cf and travels the ring i -> i+1 -> ..."""
    edges = np.asarray([(i, (i + 1) % V) for i in range(V)], dtype=np.int64)
    C = V * cf
    pre = np.zeros((C, V), dtype=np.int64)
    moves = []
    for c in range(C):
        o = c // cf
        pre[c, o] = 1
        for h in range(V - 1):
            moves.append((h, c, (o + h) % V))
    return edges, pre, _sched(V - 1, C, V, moves)


@pytest.mark.parametrize("instances,fusion", [(1, False), (2, False), (1, True), (3, True)])
def test_ring_allgather_lowers_and_checks(instances, fusion):
    edges, pre, sched = _ring_allgather(4, 2)
    xml = X.schedule_to_msccl_xml(sched, edge_src=edges[:, 0], edge_dst=edges[:, 1], pre_condition=pre,
                                  collective="allgather", instances=instances, instr_fusion=fusion)
    root = ET.fromstring(xml)
    assert root.get("coll") == "allgather" and int(root.get("ngpus")) == 4
    assert int(root.get("nchannels")) == instances and int(root.get("nchunksperloop")) == 8 * instances
    kinds = [s.get("type") for s in root.iter("step")]
    if fusion:
        assert "rcs" in kinds  # a ring relay forwards what it just received
    else:
        assert kinds.count("s") == kinds.count("r") == 4 * 2 * 3 * instances


def test_switch_deliveries_are_traced_back_to_the_injecting_gpu():
    # GPUs 0, 1, 2 and a switch 3: GPU -> switch -> GPU takes two slots
    edges = np.asarray([(0, 3), (1, 3), (2, 3), (3, 0), (3, 1), (3, 2)], dtype=np.int64)
    sw = np.asarray([False, False, False, True])
    pre = np.zeros((3, 4), dtype=np.int64)
    pre[[0, 1, 2], [0, 1, 2]] = 1
    moves = []
    for c in range(3):
        moves.append((2 * c, c, c))              # GPU c -> switch at slot 2c
        for d in range(3):
            if d != c:
                moves.append((2 * c + 1, c, 3 + d))  # switch -> GPU d at slot 2c+1
    sched = _sched(6, 3, 6, moves)
    rounds = X.gpu_transfers(sched, edges[:, 0], edges[:, 1], pre, sw)
    assert rounds[0] == [(0, 1, 0), (0, 2, 0)] and rounds[1] == []  # placed at the GPU's send slot
    xml = X.schedule_to_msccl_xml(sched, edge_src=edges[:, 0], edge_dst=edges[:, 1], pre_condition=pre,
                                  is_switch=sw, collective="allgather")
    assert int(ET.fromstring(xml).get("ngpus")) == 3
    # a switch cannot forward in the slot it receives
    bad = _sched(2, 3, 6, [(0, 0, 0), (0, 0, 4)])
    with pytest.raises(ValueError):
        X.gpu_transfers(bad, edges[:, 0], edges[:, 1], pre, sw)


@pytest.mark.parametrize("fusion", [False, True])
def test_alltoall_relays_through_scratch(fusion):
    # line 0 <-> 1 <-> 2: chunks between 0 and 2 relay on GPU 1
    edges = np.asarray([(0, 1), (1, 2), (1, 0), (2, 1)], dtype=np.int64)
    V, cf = 3, 1
    C = V * V * cf
    pre = np.zeros((C, V), dtype=np.int64)
    post = np.zeros((C, V), dtype=np.int64)
    moves = []
    route = {(0, 1): [0], (1, 2): [1], (1, 0): [2], (2, 1): [3], (0, 2): [0, 1], (2, 0): [3, 2]}
    for s in range(V):
        for d in range(V):
            c = s * V + d
            pre[c, s] = 1
            post[c, d] = 1
            for h, e in enumerate(route.get((s, d), [])):
                moves.append((h, c, e))
    sched = _sched(2, C, 4, moves)
    xml = X.schedule_to_msccl_xml(sched, edge_src=edges[:, 0], edge_dst=edges[:, 1], pre_condition=pre,
                                  post_condition=post, collective="alltoall", instr_fusion=fusion, instances=2)
    root = ET.fromstring(xml)
    assert root.get("coll") == "alltoall"
    assert any(int(g.get("s_chunks")) > 0 for g in root.iter("gpu")) or fusion


def test_check_reports_a_deadlock_and_a_wrong_slot():
    xml = ('<algo name="x" proto="Simple" nchannels="1" nchunksperloop="1" ngpus="2" coll="custom" inplace="0">'
           '<gpu id="0" i_chunks="1" o_chunks="1" s_chunks="0"><tb id="0" send="-1" recv="1" chan="0">'
           '<step s="0" type="r" srcbuf="o" srcoff="0" dstbuf="o" dstoff="0" cnt="1" depid="-1" deps="-1" hasdep="0"/>'
           '</tb></gpu><gpu id="1" i_chunks="1" o_chunks="1" s_chunks="0"></gpu></algo>')
    with pytest.raises(ValueError, match="deadlock"):
        X.check_xml(xml, lambda r, i, k: None, lambda r, i, k: (r, i))
    edges, pre, sched = _ring_allgather(3, 1)
    good = X.schedule_to_msccl_xml(sched, edge_src=edges[:, 0], edge_dst=edges[:, 1], pre_condition=pre,
                                   collective="allgather")
    with pytest.raises(ValueError, match="wrong chunk"):
        X.check_xml(good, lambda r, i, k: ("c", (i + 1) % 3, k), lambda r, i, k: ("c", r + i, k))


def test_single_problem_builders_and_cli(tmp_path):
    from revealaiccl_b200.models.policy import SlotLevelPolicy
    from revealaiccl_b200.rl import single_problem as S
    from revealaiccl_b200.topology.loader import ensure_bundled, load_topology_info

    ensure_bundled()
    topo = load_topology_info("Rear4GPU")
    ag = S.allgather_problem(topo, 2, 12)
    assert ag.C == 8 and ag.demands.sum() == 8 * 3 and (ag.initial_state.sum(axis=1) == 1).all()
    a2a = S.alltoall_problem(topo, 1, 12)
    assert a2a.C == 16 and a2a.demands.sum() == 12
    bc = S.broadcast_problem(topo, 3, root_node=2, T=12)
    assert (bc.initial_state[:, 2] == 1).all() and bc.demands[:, 2].sum() == 0
    assert S.allreduce_problem(topo, 1, 12).scenario_type == "allreduce"
    torch.manual_seed(0)
    ck = tmp_path / "m.pth"
    torch.save({"model_state_dict": SlotLevelPolicy(5, 2, 5, 2, 32).state_dict()}, ck)
    for coll in ("allgather", "alltoall", "broadcast"):
        out = tmp_path / coll
        S.main(["--model_path", str(ck), "--topology", "Rear4GPU", "--collective", coll, "--chunk_factor", "1",
                "--time_limit", "16", "--output_dir", str(out), "--export_xml", "--hidden_dim", "32"])
        summary = json.loads((out / "test_summary.json").read_text())
        assert summary["collective"] == coll and (out / f"strategy_Rear4GPU_{coll}_cf1.txt").exists()
        if coll != "broadcast":
            assert "xml_file" in summary or "xml_error" in summary

"""Schedule-search RL stack: checkpoint-compatible policy layout, decoder,
batched PPO replay identity, GAE, evaluator, scenario cache and XML export
(reference tests test_moment_policy_shapes.py, test_optimizer_checkpoint.py,
test_problem_unification.py re-expressed)."""

import json
import xml.etree.ElementTree as ET

import numpy as np
import pytest
import torch

from revealaiccl_b200.models.policy import SlotLevelPolicy
from revealaiccl_b200.rl.cli import load_checkpoint, model_name_for, save_checkpoint
from revealaiccl_b200.rl.decoder import SlotDecoder, recompute_logp_slot, rollout
from revealaiccl_b200.rl.ppo import compute_gae_advantages, evaluate_model, get_config, train_epoch
from revealaiccl_b200.rl.scenarios import (build_problem_from_scenario, evaluate_schedule, generate_scenarios,
                                           load_or_generate_scenarios)
from revealaiccl_b200.rl.xml_export import build_xml
from revealaiccl_b200.topology import ensure_bundled, load_topology_info


@pytest.fixture(scope="module")
def topo():
    ensure_bundled()
    return load_topology_info("Rear4GPU")


def _problems(topo, n=6, seed=3, T=12):
    return [(f"p{s['id']}", build_problem_from_scenario(topo.V, topo.E, topo.edges, topo.capacities,
                                                       topo.shared_constraints, s, T=T, topology_info=topo))
            for s in generate_scenarios(topo.V, n, seed)]


def test_policy_state_dict_layout_and_dims():
    m = SlotLevelPolicy(5, 2, 5, 2, 64)
    keys = set(m.state_dict())
    for k in ("node_encoder.weight", "edge_encoder.weight", "chunk_encoder.0.weight", "chunk_encoder.1.weight",
              "layer1.edge_update.0.weight", "layer1.edge_update.1.weight", "layer2.node_update.0.weight",
              "global_pool.0.weight", "actor.0.weight", "actor.2.weight", "critic.2.bias"):
        assert k in keys
    assert not any(k.startswith(("moment_encoder", "context_fusion")) for k in keys)
    assert m.actor[0].in_features == 4 * 64 + 5 + 64
    mm = SlotLevelPolicy(12, 2, 9, 2, 64, global_moment_feat_dim=8)
    assert "moment_encoder.network.0.weight" in mm.state_dict() and "context_fusion.0.weight" in mm.state_dict()
    with pytest.raises(RuntimeError):
        m.load_state_dict(mm.state_dict(), strict=True)


def test_decode_and_batched_replay_logp_identity(topo):
    torch.manual_seed(0)
    model = SlotLevelPolicy(5, 2, 5, 2, 32)
    prob = _problems(topo)[0][1]
    dec = SlotDecoder(topo)
    Y, logp, ent, value, info, micro = dec.decode_slot(model, prob.initial_state.copy(), prob.demands.copy(), 0,
                                                       prob.T, train=True)
    assert Y.shape == (prob.C, prob.E) and len(micro) == int(Y.sum())
    assert np.all(Y.sum(axis=0) <= np.asarray(topo.capacities) + 1e-6)
    logp2, ent2, value2 = recompute_logp_slot(model, info, micro, torch.device("cpu"), dec.get_static_info())
    torch.testing.assert_close(logp2, logp, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(value2, value)


def test_rollout_schedule_is_legal(topo):
    torch.manual_seed(1)
    model = SlotLevelPolicy(5, 2, 5, 2, 32)
    for _, prob in _problems(topo, 4):
        sched, done = rollout(SlotDecoder(topo), model, prob, train=False)
        score, err = evaluate_schedule(sched, prob)
        assert err == "" and score < 0


def test_evaluator_rejects_violations(topo):
    prob = _problems(topo, 1)[0][1]
    score, err = evaluate_schedule([np.ones((prob.C, prob.E), dtype=int)], prob)
    assert err and score == -(prob.T + 2)


def test_gae_matches_manual():
    r = torch.tensor([1.0, 0.0, -1.0])
    v = torch.tensor([0.5, 0.25, 0.1])
    d = torch.tensor([0.0, 0.0, 1.0])
    adv, ret = compute_gae_advantages(r, v, d, 0.9, 0.8)
    g2 = -1.0 - 0.1
    g1 = 0.0 + 0.9 * 0.1 - 0.25 + 0.9 * 0.8 * g2
    g0 = 1.0 + 0.9 * 0.25 - 0.5 + 0.9 * 0.8 * g1
    raw = torch.tensor([g0, g1, g2])
    torch.testing.assert_close(ret, raw + v)
    torch.testing.assert_close(adv, (raw - raw.mean()) / (raw.std() + 1e-8))


def test_train_epoch_and_checkpoint_roundtrip(topo, tmp_path):
    torch.manual_seed(2)
    cfg = get_config()
    cfg.update(batch_target=12, ppo_epochs=1, mini_batch_size=4, hidden_dim=32)
    model = SlotLevelPolicy(5, 2, 5, 2, 32)
    opt = torch.optim.Adam(model.parameters(), lr=cfg["lr"])
    probs = _problems(topo, 6)
    out = train_epoch(model, opt, probs, torch.device("cpu"), cfg, 0, 1, seed=0, log=lambda *a: None)
    assert all(np.isfinite(out))
    path = tmp_path / f"{model_name_for(['Rear4GPU'])}_best.pth"
    save_checkpoint(str(path), epoch=3, model=model, optimizer=opt, best_score=-5.0, config=cfg, topologies=["Rear4GPU"])
    ck = torch.load(path, weights_only=False)
    assert set(ck) == {"epoch", "model_state_dict", "optimizer_state_dict", "best_score", "config", "topologies"}
    m2 = SlotLevelPolicy(5, 2, 5, 2, 32)
    o2 = torch.optim.Adam(m2.parameters(), lr=cfg["lr"])
    assert load_checkpoint(str(path), m2, o2) == (4, -5.0)
    for a, b in zip(model.state_dict().values(), m2.state_dict().values()):
        assert torch.equal(a, b)
    torch.save(model.state_dict(), tmp_path / "bare.pth")
    assert load_checkpoint(str(tmp_path / "bare.pth"), SlotLevelPolicy(5, 2, 5, 2, 32)) == (0, -float("inf"))
    score, steps = evaluate_model(model, probs[:2], torch.device("cpu"), log=lambda *a: None)
    assert np.isfinite(score) and steps > 0


def test_scenario_cache_regenerates_on_stale_hash(tmp_path):
    p = tmp_path / "cache.json"
    a = load_or_generate_scenarios(str(p), 4, 10, 7)
    assert load_or_generate_scenarios(str(p), 4, 10, 7) == a
    data = json.loads(p.read_text())
    data["generator_config_hash"] = "stale"
    data["scenarios"] = []
    p.write_text(json.dumps(data))
    assert load_or_generate_scenarios(str(p), 4, 10, 7) == a
    assert json.loads(p.read_text())["schema_version"] == 2
    assert {s["type"] for s in a} == {"all_to_all_v", "allgather", "alltoall"}


def test_xml_export_well_formed(topo):
    torch.manual_seed(3)
    model = SlotLevelPolicy(5, 2, 5, 2, 32)
    prob = _problems(topo, 3)[0][1]
    sched, _ = rollout(SlotDecoder(topo), model, prob, train=False)
    root = ET.fromstring(build_xml(prob, sched))
    assert root.tag == "algo" and int(root.get("ngpus")) == topo.V
    sends = sum(1 for s in root.iter("step") if s.get("type") == "s")
    recvs = sum(1 for s in root.iter("step") if s.get("type") == "r")
    assert sends == recvs == int(sum(int(np.asarray(Y).sum()) for Y in sched))

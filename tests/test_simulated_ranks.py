"""CPU simulated-ranks run of the progressive MoE layer (no GPU).

Two logical ranks in one process on a 2-GPU NVSwitch control projection; 4
experts (2 per rank), 1024 tokens per rank, hidden 256 fp32 with N(0,1)
activations, router weights N(0, 0.02), seeded top-2 over 8 chunks of 128.
Checks static / single-step / trajectory equivalence of the compiled
scheduler with the uncompiled one, zero unrevealed commits, every token
dispatched and returned exactly once, Early == Delayed outputs, and that a
hidden (unrevealed) future chunk cannot change any earlier commit.
"""

import numpy as np
import pytest
import torch

from revealaiccl_b200.moe.config import preset
from revealaiccl_b200.moe.simulated import SimulatedMoE
from revealaiccl_b200.ops import _native

BACKENDS = ["numpy"] + (["native"] if _native.has_host() else [])


@pytest.fixture(scope="module")
def sim():
    return SimulatedMoE(preset("cpu_sim_2rank"), world=2)


@pytest.mark.parametrize("backend", BACKENDS)
def test_two_rank_run_is_exact_and_complete(sim, backend):
    sim.backend = backend
    res = sim.run("early")
    eq = res.equivalence
    assert eq["total"] == 2 * sim.cfg.n_desc
    assert eq["static"] == eq["single_step"] == eq["trajectory"] == eq["total"]
    assert eq["runtime_bfs_calls"] == 0 and eq["full_rebuild_count"] == 0
    assert all(v == 0 for v in res.counters.values())
    assert all(c["pass"] for c in res.forward_checks)
    assert all(c["pass"] for c in res.return_checks)
    sent = sum(c["tokens"] for c in res.forward_checks)
    assert sent == 2 * sim.cfg.tokens_per_rank * sim.cfg.top_k
    assert res.transport["signals"] == res.transport["put_calls"] > 0


def test_early_equals_delayed(sim):
    a = sim.run("early")
    b = sim.run("delayed")
    for x, y in zip(a.outputs, b.outputs):
        assert torch.equal(x, y)
    assert a.actions == b.actions


def test_hidden_future_perturbation_cannot_change_committed_actions(sim):
    base = sim.run("early")
    cfg = sim.cfg
    rng = np.random.default_rng(7)
    cut = cfg.progressive_chunks // 2
    routes = []
    for ids, gates, logits in sim.route:
        ids2 = ids.clone()
        lo = cfg.chunk_offsets[cut + 1]
        perm = torch.from_numpy(rng.permutation(cfg.experts)).to(torch.int32)
        ids2[lo:] = perm[ids2[lo:].long()]
        routes.append((ids2, gates, logits))
    sim2 = SimulatedMoE.__new__(SimulatedMoE)
    sim2.__dict__.update(sim.__dict__)
    eq = {"static": 0, "single_step": 0, "trajectory": 0, "total": 0, "runtime_bfs_calls": 0, "full_rebuild_count": 0}
    for r in range(sim.world):
        _, acts = sim2.run_control(r, routes[r][0].numpy(), eq)
        assert acts[:cut + 1] == base.actions[r][:cut + 1]
    assert eq["trajectory"] == eq["total"]

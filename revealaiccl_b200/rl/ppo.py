"""PPO training of the slot-level schedule policy (rlccl/training/ppo_trainer.py,
rlccl/training/buffer.py).

Slot reward = -remaining demand / initial demand; GAE advantages (normalised);
clipped surrogate + value MSE - entropy bonus; per-slot log-probabilities are
recomputed by batched replay (``recompute_logp_slot``); gradient clipping.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from ..topology.info import compute_received_chunks
from .decoder import SlotDecoder, recompute_logp_slot, rollout
from .scenarios import evaluate_schedule

DEFAULT_TRAIN_CONFIG = {
    "epochs": 30, "ppo_epochs": 10, "batch_target": 500, "lr": 3e-4, "hidden_dim": 128, "gamma": 0.99,
    "gae_lambda": 0.95, "clip_eps": 0.2, "entropy_coef": 0.01, "value_coef": 0.5, "mini_batch_size": 16,
    "max_grad_norm": 0.5,
}


def get_config() -> dict:
    return dict(DEFAULT_TRAIN_CONFIG)


class SlotBuffer:
    """Slot-level experience (static topology info is shared, not copied)."""

    def __init__(self) -> None:
        self.clear()

    def clear(self) -> None:
        self.slot_states, self.slot_actions, self.slot_logprobs = [], [], []
        self.slot_values, self.slot_rewards, self.slot_dones, self.slot_static_infos = [], [], [], []

    def add(self, state_info, actions, logprob_slot, value, reward, done, static_info=None) -> None:
        self.slot_states.append(state_info)
        self.slot_actions.append(actions)
        self.slot_logprobs.append(logprob_slot)
        self.slot_values.append(value)
        self.slot_rewards.append(reward)
        self.slot_dones.append(done)
        self.slot_static_infos.append(static_info)

    def __len__(self) -> int:
        return len(self.slot_rewards)


def compute_gae_advantages(rewards, values, dones, gamma, gae_lambda):
    adv = []
    gae = 0.0
    for t in reversed(range(len(rewards))):
        if dones[t]:
            gae, nxt = 0.0, 0.0
        else:
            nxt = values[t + 1].item() if t + 1 < len(values) else 0.0
        delta = rewards[t] + gamma * nxt - values[t]
        gae = delta + gamma * gae_lambda * gae
        adv.insert(0, gae)
    adv = torch.tensor(adv, dtype=torch.float32)
    ret = adv + values
    if len(adv) > 1:
        adv = (adv - adv.mean()) / (adv.std() + 1e-8)
    return adv, ret


def collect(model, problems, config, rng) -> SlotBuffer:
    buf = SlotBuffer()
    got = 0
    for i in rng.permutation(len(problems)):
        if got >= config["batch_target"]:
            break
        _, prob = problems[i]
        if np.sum(prob.demands) == 0 or getattr(prob, "topology_info", None) is None:
            continue
        dec = SlotDecoder(prob.topology_info)
        static = dec.get_static_info()
        state, demands = prob.initial_state.copy(), prob.demands.copy()
        total = max(1.0, float(np.sum(prob.demands)))
        for t in range(prob.T):
            Y, logp, _, value, info, micro = dec.decode_slot(
                model, state, demands, t, prob.T, train=True,
                moment_context=(getattr(prob, "moment_context", None)
                                if getattr(model, "global_moment_feat_dim", 0) > 0 else None),
                current_matrix=getattr(prob, "traffic_matrix", None),
                moment_max_entry=config.get("moment_max_entry", 8.0))
            N = compute_received_chunks(Y, prob.topology_info.edge_dst, prob.topology_info.V)
            state = np.maximum(state, N)
            demands = demands * (1 - N)
            end = bool(np.sum(demands) == 0 or t == prob.T - 1)
            buf.add(info, micro, logp.detach().cpu(), value.detach().cpu(), -float(np.sum(demands)) / total, end, static)
            got += 1
            if end:
                break
    return buf


def train_epoch(model, optimizer, train_problems, device, config, epoch, total_epochs, *, seed=None, log=print):
    model.train()
    rng = np.random.default_rng(seed) if seed is not None else np.random.default_rng()
    buf = collect(model, train_problems, config, rng)
    if len(buf) == 0:
        log("  No slots collected, skipping update")
        return 0.0, 0.0, 0.0, 0.0
    rewards = torch.tensor(buf.slot_rewards, dtype=torch.float32)
    values = torch.tensor([v.item() for v in buf.slot_values], dtype=torch.float32)
    dones = torch.tensor(buf.slot_dones, dtype=torch.float32)
    adv, ret = compute_gae_advantages(rewards, values, dones, config["gamma"], config["gae_lambda"])
    n = len(buf)
    order = np.arange(n)
    tp = tv = te = 0.0
    updates = 0
    for _ in range(config["ppo_epochs"]):
        rng.shuffle(order)
        for s in range(0, n, config["mini_batch_size"]):
            idx = order[s:s + config["mini_batch_size"]]
            optimizer.zero_grad()
            loss = 0.0
            for i in idx:
                logp, ent, v = recompute_logp_slot(model, buf.slot_states[i], buf.slot_actions[i], device,
                                                   buf.slot_static_infos[i])
                ratio = torch.exp(logp - buf.slot_logprobs[i].to(device))
                a = adv[i].to(device)
                pl = -torch.min(ratio * a, torch.clamp(ratio, 1 - config["clip_eps"], 1 + config["clip_eps"]) * a)
                vl = F.mse_loss(v.squeeze(), ret[i].to(device))
                loss = loss + pl + config["value_coef"] * vl - config["entropy_coef"] * ent
                tp += pl.item()
                tv += vl.item()
                te += ent.item()
            (loss / len(idx)).backward()
            if "max_grad_norm" in config:
                torch.nn.utils.clip_grad_norm_(model.parameters(), config["max_grad_norm"])
            optimizer.step()
            updates += len(idx)
    u = max(updates, 1)
    return tp / u, tv / u, te / u, rewards.mean().item()


def evaluate_model(model, test_problems, device, moment_max_entry=8.0, log=print):
    model.eval()
    scores, steps = [], []
    with torch.no_grad():
        for sid, prob in test_problems:
            topo = getattr(prob, "topology_info", None)
            if topo is None:
                continue
            schedule, done = rollout(SlotDecoder(topo), model, prob, train=False, moment_max_entry=moment_max_entry)
            steps.append(done)
            score, err = evaluate_schedule(schedule, prob)
            if err == "":
                scores.append(score)
            else:
                log(f"  Warning: Problem {sid} evaluation failed: {err}")
    if scores:
        return float(np.mean(scores)), float(np.mean(steps))
    return -1000.0, 0.0


__all__ = ["DEFAULT_TRAIN_CONFIG", "SlotBuffer", "collect", "compute_gae_advantages", "evaluate_model", "get_config",
           "train_epoch"]

"""Autoregressive slot decoder of the schedule-search policy
(rlccl/envs/decoder.py:118-671).

Per slot t the decoder encodes the state once with the GNN, forms every
valid (chunk, edge) candidate — the edge source holds the chunk and the edge
target lacks it — and then takes up to sum(capacity) + 5 micro-steps: mask
by remaining edge capacity, already-received (node, chunk) pairs and full
shared groups; keep at most 256 (train) / 512 (eval) candidates ranked by the
demand/distance heuristic; score them with the actor; sample (train) or
argmax (eval); commit the action into Y_t and the usage counters.  Replay
info is kept so ``recompute_logp_slot`` re-scores every micro-step of a slot
in one batched forward pass for PPO.

Feature definitions (node 5 [+7 moment], edge 2, chunk 2, candidate 5
[+4 moment], global moment 8) are part of the trained-policy contract.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F
from torch.distributions import Categorical

from ..topology.info import compute_received_chunks
from ..traffic.matrix_utils import validate_traffic_matrix

MOMENT_NODE_FEAT_DIM = 7
GLOBAL_MOMENT_FEAT_DIM = 8
CANDIDATE_MOMENT_FEAT_DIM = 4
MOMENT_Z_CLIP = 10.0
_MOMENT_NODE_KEYS = ("source_current_send_z", "destination_current_recv_z", "source_expected_send",
                     "destination_expected_recv")


def _cv(values, eps=1e-6) -> float:
    v = np.asarray(values, dtype=np.float64)
    return float(v.std(ddof=0) / (abs(v.mean()) + eps))


def get_moment_node_features(mc, z_clip=MOMENT_Z_CLIP) -> np.ndarray:
    sm, rm = np.asarray(mc.send_mean, float), np.asarray(mc.recv_mean, float)
    ss, rs = np.asarray(mc.send_std, float), np.asarray(mc.recv_std, float)
    mscale = max(float(np.mean(np.concatenate([sm, rm]))), 1e-6)
    sscale = max(float(np.mean(np.concatenate([ss, rs]))), 1e-6)
    conf = np.full_like(sm, float(mc.confidence))
    return np.stack([sm / mscale, rm / mscale, ss / sscale, rs / sscale,
                     np.clip(mc.current_send_z, -z_clip, z_clip) / z_clip,
                     np.clip(mc.current_recv_z, -z_clip, z_clip) / z_clip, conf], axis=1).astype(np.float32)


def get_candidate_moment_node_arrays(mc, z_clip=MOMENT_Z_CLIP) -> dict:
    sm, rm = np.asarray(mc.send_mean, float), np.asarray(mc.recv_mean, float)
    mscale = max(float(np.mean(np.concatenate([sm, rm]))), 1e-6)
    return {"source_current_send_z": (np.clip(mc.current_send_z, -z_clip, z_clip) / z_clip).astype(np.float32),
            "destination_current_recv_z": (np.clip(mc.current_recv_z, -z_clip, z_clip) / z_clip).astype(np.float32),
            "source_expected_send": (sm / mscale).astype(np.float32),
            "destination_expected_recv": (rm / mscale).astype(np.float32)}


def get_global_moment_features(mc, current_matrix=None, max_entry=8.0) -> np.ndarray:
    if current_matrix is not None:
        validate_traffic_matrix(current_matrix)
        m = np.asarray(current_matrix, dtype=np.float64)
        off = m[~np.eye(m.shape[0], dtype=bool)]
        sparsity = float(np.mean(off == 0)) if off.size else 1.0
        src_load, dst_load = m.sum(axis=1), m.sum(axis=0)
        mx = float(m.max()) if m.size else 0.0
    else:
        src_load = np.asarray(mc.send_mean) + np.asarray(mc.current_send_z) * np.asarray(mc.send_std)
        dst_load = np.asarray(mc.recv_mean) + np.asarray(mc.current_recv_z) * np.asarray(mc.recv_std)
        sparsity, mx = 0.0, 0.0
    return np.asarray([np.clip(mc.mean_drift, 0.0, 10.0), np.clip(mc.var_drift, 0.0, 10.0),
                       np.clip(mc.confidence, 0.0, 1.0),
                       np.clip(mc.history_length / max(mc.window_size, 1), 0.0, 1.0), sparsity,
                       _cv(src_load), _cv(dst_load), mx / max(float(max_entry), 1e-6)], dtype=np.float32)


def get_candidate_moment_features(cand_e, edge_src, edge_dst, arrays) -> np.ndarray:
    s, d = edge_src[cand_e], edge_dst[cand_e]
    return np.stack([arrays["source_current_send_z"][s], arrays["destination_current_recv_z"][d],
                     arrays["source_expected_send"][s], arrays["destination_expected_recv"][d]],
                    axis=1).astype(np.float32)


def _candidate_features(cand_c, cand_e, edge_src, edge_dst, V, caps, demands, dist_to_demand, edge_usage,
                        group_usage, edge_to_groups, group_limits, num_groups, step, max_steps) -> np.ndarray:
    s, d = edge_src[cand_e], edge_dst[cand_e]
    f_demand = demands[cand_c, d].astype(np.float32)
    f_dist = (dist_to_demand[cand_c, s] - dist_to_demand[cand_c, d]) / max(1.0, V)
    f_edge = (caps[cand_e] - edge_usage[cand_e]) / np.maximum(caps[cand_e], 1e-6)
    f_group = np.ones(len(cand_e), dtype=np.float32)
    if num_groups > 0:
        for i, e in enumerate(cand_e):
            gs = edge_to_groups[e]
            if gs:
                f_group[i] = min(1.0, min((group_limits[g] - group_usage[g]) / max(group_limits[g], 1e-6) for g in gs))
    f_step = np.full(len(cand_e), step / max(max_steps, 1), dtype=np.float32)
    return np.stack([f_demand, f_dist, f_edge, f_group, f_step], axis=1).astype(np.float32)


class SlotDecoder:
    def __init__(self, topology_info):
        self.topo = topology_info
        self.V, self.E = int(topology_info.V), int(topology_info.E)
        self.edge_src = np.asarray(topology_info.edge_src, dtype=np.int64)
        self.edge_dst = np.asarray(topology_info.edge_dst, dtype=np.int64)
        self.capacities = np.asarray(topology_info.capacities, dtype=np.float32)
        dist = getattr(topology_info, "dist_matrix", None)
        if dist is None:
            from ..topology.info import hop_distances

            dist = hop_distances(self.V, np.stack([self.edge_src, self.edge_dst], axis=1))
        self.dist_matrix = np.asarray(dist, dtype=np.float32)
        self.group_to_edges, self.edge_to_groups, limits = [], [[] for _ in range(self.E)], []
        for g, (edges, limit) in enumerate(getattr(topology_info, "shared_constraints", []) or []):
            self.group_to_edges.append(np.asarray(edges, dtype=np.int64))
            limits.append(float(limit))
            for e in edges:
                self.edge_to_groups[e].append(g)
        self.group_limits = np.asarray(limits, dtype=np.float32) if limits else np.array([1.0], dtype=np.float32)
        self.num_groups = len(self.group_to_edges)
        out_deg = np.zeros(self.V, dtype=np.float32)
        in_deg = np.zeros(self.V, dtype=np.float32)
        np.add.at(out_deg, self.edge_src, 1)
        np.add.at(in_deg, self.edge_dst, 1)
        self.f_out, self.f_in = out_deg / max(1, self.E), in_deg / max(1, self.E)
        self.max_steps = int(self.capacities.sum()) + 5
        self.edge_src_t = torch.tensor(self.edge_src, dtype=torch.long)
        self.edge_dst_t = torch.tensor(self.edge_dst, dtype=torch.long)
        self._static = {"edge_src_t": self.edge_src_t.clone(), "edge_dst_t": self.edge_dst_t.clone(),
                        "capacities": self.capacities.copy(), "max_steps": self.max_steps,
                        "group_limits": self.group_limits.copy(), "edge_to_groups": self.edge_to_groups,
                        "num_groups": self.num_groups, "V": self.V, "E": self.E}

    def get_static_info(self) -> dict:
        return self._static

    def compute_dist_to_demand(self, demands: np.ndarray) -> np.ndarray:
        C, V = demands.shape
        out = np.full((C, V), V + 1.0, dtype=np.float32)
        for v in range(V):
            cs = np.flatnonzero(demands[:, v])
            if cs.size:
                out[cs, :] = np.minimum(out[cs, :], self.dist_matrix[:, v])
        return out

    def get_node_features(self, state, demands, t, T) -> np.ndarray:
        C, V = state.shape
        return np.stack([state.sum(axis=0) / max(1, C), demands.sum(axis=0) / max(1, C), self.f_out, self.f_in,
                         np.full(V, t / max(1, T), dtype=np.float32)], axis=1).astype(np.float32)

    def get_chunk_features(self, state, demands) -> np.ndarray:
        _, V = state.shape
        return np.stack([1.0 - state.sum(axis=1) / max(1, V), demands.sum(axis=1) / max(1, V)],
                        axis=1).astype(np.float32)

    def get_edge_features(self, edge_usage) -> np.ndarray:
        return np.stack([(self.capacities - edge_usage) / np.maximum(self.capacities, 1e-6),
                         self.capacities / max(float(np.max(self.capacities)), 1e-6)], axis=1).astype(np.float32)

    def get_candidate_dynamic_features(self, cand_c, cand_e, demands, dist_to_demand, edge_usage, group_usage,
                                       step, max_steps) -> np.ndarray:
        return _candidate_features(cand_c, cand_e, self.edge_src, self.edge_dst, self.V, self.capacities, demands,
                                   dist_to_demand, edge_usage, group_usage, self.edge_to_groups, self.group_limits,
                                   self.num_groups, step, max_steps)

    def decode_slot(self, model, state, demands, t, T, train=True, moment_context=None, current_matrix=None,
                    moment_max_entry=8.0, observation_demands=None):
        device = next(model.parameters()).device
        C, V = state.shape
        E = self.E
        pd = demands if observation_demands is None else np.asarray(observation_demands, dtype=np.float32)
        if pd.shape != demands.shape:
            raise ValueError("observation_demands must have the same chunk/node shape as demands")
        if not np.all(np.isfinite(pd)) or np.any(pd < 0):
            raise ValueError("observation_demands must be finite and nonnegative")
        if self.edge_src_t.device != device:
            self.edge_src_t, self.edge_dst_t = self.edge_src_t.to(device), self.edge_dst_t.to(device)
        dist_to_demand = self.compute_dist_to_demand(pd)
        node_np = self.get_node_features(state, pd, t, T)
        chunk_np = self.get_chunk_features(state, pd)
        edge_np = self.get_edge_features(np.zeros(E, dtype=np.float32))
        moment = getattr(model, "global_moment_feat_dim", 0) > 0
        gm_np = cand_arrays = node_m = None
        if moment:
            if moment_context is None:
                node_m = np.zeros((V, MOMENT_NODE_FEAT_DIM), dtype=np.float32)
                gm_np = np.zeros(GLOBAL_MOMENT_FEAT_DIM, dtype=np.float32)
                cand_arrays = {k: np.zeros(V, dtype=np.float32) for k in _MOMENT_NODE_KEYS}
            else:
                node_m = get_moment_node_features(moment_context)
                gm_np = get_global_moment_features(moment_context, current_matrix, moment_max_entry)
                cand_arrays = get_candidate_moment_node_arrays(moment_context)
            node_np = np.concatenate([node_np, node_m], axis=1)
        want = getattr(model, "node_feat_dim", node_np.shape[1])
        if node_np.shape[1] != want:
            raise ValueError(f"Decoder produced {node_np.shape[1]} node features, model expects {want}")
        node_f = torch.tensor(node_np, dtype=torch.float32, device=device)
        chunk_f = torch.tensor(chunk_np, dtype=torch.float32, device=device)
        edge_f = torch.tensor(edge_np, dtype=torch.float32, device=device)
        gm = torch.tensor(gm_np, dtype=torch.float32, device=device) if gm_np is not None else None
        with torch.no_grad():
            h_v, h_e, h_c, g_ctx = model.encode_state(node_f, edge_f, self.edge_src_t, self.edge_dst_t, chunk_f,
                                                      global_moment_feats=gm)
            value = model.get_value(g_ctx)
        valid = (state[:, self.edge_src] == 1) & ((1 - state[:, self.edge_dst]) == 1)
        all_c, all_e = np.nonzero(valid)
        info = {"node_feats": node_f.cpu(), "edge_feats": edge_f.cpu(), "chunk_feats": chunk_f.cpu(),
                "demands": pd.copy(), "dist_to_demand": dist_to_demand.copy(), "moment_enabled": moment,
                "global_moment_feats": gm.cpu() if gm is not None else None,
                "node_moment_feats": node_m.copy() if node_m is not None else None,
                "candidate_moment_node_arrays": ({k: v.copy() for k, v in cand_arrays.items()}
                                                 if cand_arrays is not None else None)}
        Y = np.zeros((C, E), dtype=int)
        if all_c.size == 0:
            z = torch.tensor(0.0, device=device)
            return Y, z, z.clone(), value, info, []
        edge_usage = np.zeros(E, dtype=np.float32)
        group_usage = np.zeros(self.num_groups, dtype=np.float32)
        received = np.zeros((V, C), dtype=bool)
        active = np.ones(all_c.size, dtype=bool)
        cand_dst_all = self.edge_dst[all_e]
        micro, logps, ents = [], [], []
        for step in range(self.max_steps):
            m_edge = edge_usage[all_e] < self.capacities[all_e]
            m_recv = ~received[cand_dst_all, all_c]
            m_group = np.ones(all_c.size, dtype=bool)
            if self.num_groups > 0:
                full = group_usage >= self.group_limits
                if np.any(full):
                    blocked = np.zeros(E, dtype=bool)
                    for g in np.flatnonzero(full):
                        blocked[self.group_to_edges[g]] = True
                    m_group = ~blocked[all_e]
            cur = active & m_edge & m_recv & m_group
            if not np.any(cur):
                break
            idx = np.flatnonzero(cur)
            cap = 256 if train else 512
            if idx.size > cap:
                ac, ae = all_c[idx], all_e[idx]
                score = demands[ac, self.edge_dst[ae]].astype(np.float32) * 10.0 + \
                    (dist_to_demand[ac, self.edge_src[ae]] - dist_to_demand[ac, self.edge_dst[ae]]) / max(1.0, self.V)
                idx = idx[np.argsort(score)[-cap:]]
            cc, ce = all_c[idx], all_e[idx]
            feats = self.get_candidate_dynamic_features(cc, ce, pd, dist_to_demand, edge_usage, group_usage, step,
                                                        self.max_steps)
            if moment:
                feats = np.concatenate([feats, get_candidate_moment_features(ce, self.edge_src, self.edge_dst,
                                                                             cand_arrays)], axis=1)
            want_c = getattr(model, "cand_feat_dim", feats.shape[1])
            if feats.shape[1] != want_c:
                raise ValueError(f"Decoder produced {feats.shape[1]} candidate features, model expects {want_c}")
            with torch.no_grad():
                logits = model.get_candidate_logits(
                    h_v, h_e, h_c, g_ctx, self.edge_src_t, self.edge_dst_t,
                    torch.tensor(ce, dtype=torch.long, device=device), torch.tensor(cc, dtype=torch.long, device=device),
                    torch.tensor(feats, dtype=torch.float32, device=device))
                dist = Categorical(probs=F.softmax(logits, dim=0))
                a = dist.sample() if train else torch.argmax(logits)
                logps.append(dist.log_prob(a))
                ents.append(dist.entropy())
            i = int(a.item())
            g_i = idx[i]
            c, e, v = all_c[g_i], all_e[g_i], cand_dst_all[g_i]
            micro.append({"action_idx": i, "cand_c": cc.copy(), "cand_e": ce.copy(), "selected_e": e, "step": step})
            Y[c, e] = 1
            active[g_i] = False
            edge_usage[e] += 1
            for g in self.edge_to_groups[e]:
                group_usage[g] += 1
            received[v, c] = True
        if logps:
            return Y, torch.stack(logps).sum(), torch.stack(ents).mean(), value, info, micro
        z = torch.tensor(0.0, device=device)
        return Y, z, z.clone(), value, info, micro


def recompute_logp_slot(model, state_info, micro_actions, device, static_info):
    """Re-score every micro-step of a slot in one batched actor pass (PPO)."""
    node_f = state_info["node_feats"].to(device)
    edge_f = state_info["edge_feats"].to(device)
    chunk_f = state_info["chunk_feats"].to(device)
    demands, d2d = state_info["demands"], state_info["dist_to_demand"]
    moment = bool(state_info.get("moment_enabled", False))
    gm = state_info.get("global_moment_feats")
    gm = gm.to(device) if gm is not None else None
    cand_arrays = state_info.get("candidate_moment_node_arrays")
    es, ed = static_info["edge_src_t"].to(device), static_info["edge_dst_t"].to(device)
    V, E, max_steps = static_info["V"], static_info["E"], static_info["max_steps"]
    caps, limits = static_info["capacities"], static_info["group_limits"]
    e2g, ng = static_info["edge_to_groups"], static_info["num_groups"]
    h_v, h_e, h_c, g_ctx = model.encode_state(node_f, edge_f, es, ed, chunk_f, global_moment_feats=gm)
    value = model.get_value(g_ctx)
    if not micro_actions:
        z = torch.tensor(0.0, device=device)
        return z, z.clone(), value
    edge_usage = np.zeros(E, dtype=np.float32)
    group_usage = np.zeros(ng, dtype=np.float32)
    es_np, ed_np = es.cpu().numpy(), ed.cpu().numpy()
    ce_all, cc_all, feats_all, sizes, taken = [], [], [], [], []
    for ma in micro_actions:
        cc, ce = ma["cand_c"], ma["cand_e"]
        f = _candidate_features(cc, ce, es_np, ed_np, V, caps, demands, d2d, edge_usage, group_usage, e2g, limits,
                                ng, ma["step"], max_steps)
        if moment:
            if cand_arrays is None:
                raise ValueError("Missing candidate moment replay arrays")
            f = np.concatenate([f, get_candidate_moment_features(ce, es_np, ed_np, cand_arrays)], axis=1)
        ce_all.append(ce)
        cc_all.append(cc)
        feats_all.append(f)
        sizes.append(len(ce))
        taken.append(ma["action_idx"])
        edge_usage[ma["selected_e"]] += 1
        for g in e2g[ma["selected_e"]]:
            group_usage[g] += 1
    logits = model.get_candidate_logits(
        h_v, h_e, h_c, g_ctx, es, ed, torch.tensor(np.concatenate(ce_all), dtype=torch.long, device=device),
        torch.tensor(np.concatenate(cc_all), dtype=torch.long, device=device),
        torch.tensor(np.concatenate(feats_all), dtype=torch.float32, device=device))
    logps, ents, off = [], [], 0
    for n, a in zip(sizes, taken):
        dist = Categorical(probs=F.softmax(logits[off:off + n], dim=0))
        off += n
        logps.append(dist.log_prob(torch.tensor(a, dtype=torch.long, device=device)))
        ents.append(dist.entropy())
    return torch.stack(logps).sum(), torch.stack(ents).mean(), value


def rollout(decoder: SlotDecoder, model, problem, *, train=False, moment_max_entry=8.0):
    """Decode every slot of a problem greedily (eval) or by sampling; returns
    (schedule, completion step)."""
    state, demands = problem.initial_state.copy(), problem.demands.copy()
    schedule, done = [], problem.T
    for t in range(problem.T):
        Y = decoder.decode_slot(model, state, demands, t, problem.T, train=train,
                                moment_context=(getattr(problem, "moment_context", None)
                                                if getattr(model, "global_moment_feat_dim", 0) > 0 else None),
                                current_matrix=getattr(problem, "traffic_matrix", None),
                                moment_max_entry=moment_max_entry)[0]
        schedule.append(Y)
        N = compute_received_chunks(Y, decoder.edge_dst, decoder.V)
        state = np.maximum(state, N)
        demands = demands * (1 - N)
        if np.sum(demands) == 0:
            done = t + 1
            break
    while len(schedule) < problem.T:
        schedule.append(np.zeros((problem.C, problem.E), dtype=int))
    return schedule, done


__all__ = ["CANDIDATE_MOMENT_FEAT_DIM", "GLOBAL_MOMENT_FEAT_DIM", "MOMENT_NODE_FEAT_DIM", "SlotDecoder",
           "get_candidate_moment_features", "get_candidate_moment_node_arrays", "get_global_moment_features",
           "get_moment_node_features", "recompute_logp_slot", "rollout"]

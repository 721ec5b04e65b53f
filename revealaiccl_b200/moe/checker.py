"""Fail-closed post-hoc checker of a ProgressiveMoELayer call (untimed).

Counters follow the reference gate of scripts/run_r4_a0_c0_full_moe.py:842-932
and the verifiers of rlccl/transport/reference_full_moe.py:101-246:

forward (at every expert rank, over every received row)
    duplicate, wrong_source, wrong_destination, wrong_expert, corruption
    (identity checksum and the row digest recomputed over the received bytes)
return (at every source rank, over every (token, choice) row)
    lost, wrong_destination, wrong_return, wrong_position, wrong_expert,
    corruption, expert_output_mismatch (vs the fp32 oracle)
final
    combined output vs the oracle; revealed-only packing counters
    (future / unrevealed / duplicate / stale) all zero; every descriptor
    permitted in this call
control
    differential replay of the device control-plane log: at every trigger the
    device's candidates and selection must equal the compiled scheduler's and
    the uncompiled planner's, and its guard verdict / applied count / version
    must equal the trusted checker's on an append-only oracle world.
"""

from __future__ import annotations

from typing import Any

import numpy as np
import torch

from ..scheduling.compiled import DynamicGuard, FastBinder, IncrementalState, structural_signature
from ..scheduling.recourse import bind_action
from ..scheduling.robust_prefix import build_scheduling_view, enumerate_candidates, pack_candidate_batch
from ..topology.info import TopologyInfo
from ..transport.formats import identity_checksum_vec
from ..uncertainty.execution import Proposal, commit_proposal
from ..uncertainty.observation import PartialObservationState, RevealedDemandToken, TruthTokenId
from ..uncertainty.problem import UncertainProblemInstance
from .oracle import layer_reference, router_logits

LOG_HEADER = 16  # 8-word decision record + 8 phase-clock words


class CheckerFailure(RuntimeError):
    def __init__(self, report: dict):
        self.report = report
        super().__init__(f"MoE layer check failed: {report}")


class OracleWorld:
    """Append-only trusted world holding the control-projection tokens under the
    runtime's opaque ids (scripts/run_r2_f0_integrated.py:133-205 semantics)."""

    def __init__(self, topology: TopologyInfo, sequence_id: str) -> None:
        n = int(topology.V)
        self.world = UncertainProblemInstance.from_traffic_matrix(
            truth_matrix=np.zeros((n, n), dtype=np.int64), topology_info=topology, time_limit=128,
            sequence_id=sequence_id, sequence_step=8, family="moe-control-projection",
            generator_metadata={})
        self.tokens: list[RevealedDemandToken] = []

    def append(self, tokens) -> None:
        w = self.world
        atomic = list(w._atomic)
        rows = []
        for tok in tokens:
            pair = (int(tok.source), int(tok.destination))
            private = len(atomic)
            atomic.append((pair[0], pair[1], len(w._pair_indices[pair])))
            w._pair_indices[pair].append(private)
            w._truth[pair] += 1
            row = np.zeros(w._truth.shape[0], dtype=bool)
            row[pair[0]] = True
            rows.append(row)
            w._public_to_private[tok.token_id] = private
            w._private_to_public[private] = tok.token_id
            self.tokens.append(tok)
        w._atomic = tuple(atomic)
        if rows:
            vals = np.asarray(rows, dtype=bool)
            w._possession = vals if w._possession.shape[0] == 0 else np.vstack((w._possession, vals))

    def observation(self, *, stage: int, ratio: float, final: bool) -> PartialObservationState:
        w = self.world
        n = w._truth.shape[0]
        cur = tuple(RevealedDemandToken(t.token_id, t.source, t.destination,
                                        tuple(int(v) for v in np.flatnonzero(w._possession[w._public_to_private[t.token_id]])))
                    for t in self.tokens)
        observed = np.zeros((n, n), dtype=np.int64)
        for t in cur:
            observed[t.source, t.destination] += 1
        entry = np.ones((n, n), dtype=bool) if final else np.eye(n, dtype=bool)
        return PartialObservationState(
            sequence_id=w.sequence_id, sequence_step=w.sequence_step, family=w.family,
            mode="partial_shards", stage=int(stage), ratio=float(ratio), entry_mask=entry,
            observed_matrix=observed, unknown_mask=~entry, revealed_tokens=cur, source_totals=None,
            destination_totals=None, topology=w.public_topology, state_version=w._state_version)


def control_tokens(layer, ids: np.ndarray, chunk: int, token_ids: np.ndarray) -> list[RevealedDemandToken]:
    cfg = layer.cfg
    off = cfg.chunk_offsets
    out = []
    for i in range(min(cfg.ctl_per_chunk, off[chunk + 1] - off[chunk])):
        pos = off[chunk] + i
        src = pos % cfg.ctl_nodes
        dst = int(ids[pos, 0]) % cfg.ctl_nodes
        if src == dst:
            continue
        out.append(RevealedDemandToken(TruthTokenId(f"moe:{cfg.name}:rank{layer.rank}:token{int(token_ids[pos])}"),
                                       src, dst, (src,)))
    return out


def replay_control(layer, ids: np.ndarray, token_ids: np.ndarray, log: np.ndarray) -> dict[str, int]:
    cfg = layer.cfg
    plan = layer.plan
    topo = TopologyInfo(plan.nodes, len(plan.edges), np.asarray(plan.edges), np.asarray(plan.capacity_units, dtype=float),
                        [(list(m), float(l)) for m, l in zip(plan.group_edges, plan.group_limits)])
    oracle = OracleWorld(topo, f"moe-{cfg.name}-rank{layer.rank}")
    state = IncrementalState(plan, max_tokens=layer.max_ctl_tokens, max_chunks=max(8, cfg.chunks),
                             sequence_id="", sequence_step=8)
    binder, guard = FastBinder(plan, backend="numpy"), DynamicGuard(plan, backend="numpy")
    P, C = cfg.progressive_chunks, cfg.chunks
    div = {"device_candidate_divergences": 0, "device_action_divergences": 0, "candidate_divergences": 0,
           "action_divergences": 0, "checker_divergences": 0, "holder_divergences": 0, "legal": 0, "total": 0}
    for d, group in enumerate(cfg.descriptor_groups):
        toks_by_chunk = {c: control_tokens(layer, ids, c, token_ids) for c in group}
        for c in group:
            state.stage_ready_chunk(c, toks_by_chunk[c])
        for c in group:
            state.consume_pending_chunk(c)
            oracle.append(toks_by_chunk[c])
        final = d >= P
        state.stage, state.ratio = (C, 1.0) if final else (d + 1, (d + 1) / C)
        bound = binder.step(state)
        decision = guard.apply(state, bound.proposal, require_scheduler_semantics=True,
                               expected_state_version=bound.state_version)
        rec = log[d]
        n, kept = int(rec[0]), int(rec[1])
        dev_sel = tuple((int(rec[LOG_HEADER + 2 * i]), int(rec[LOG_HEADER + 2 * i + 1])) for i in range(kept))
        cbase = LOG_HEADER + 2 * layer.max_ctl_tokens
        dev_cand = tuple(tuple(int(v) for v in rec[cbase + 4 * i: cbase + 4 * i + 4]) for i in range(min(n, layer.max_cands)))
        div["device_candidate_divergences"] += int(dev_cand != structural_signature(bound.candidates))
        div["device_action_divergences"] += int(dev_sel != tuple((c.local_token_ordinal, c.edge_index) for c in bound.selected))
        div["checker_divergences"] += int(bool(rec[2]) != decision.accepted or int(rec[4]) != decision.applied_actions
                                          or int(rec[5]) != decision.state_version)
        obs = oracle.observation(stage=state.stage, ratio=state.ratio, final=final)
        view = build_scheduling_view(obs)
        old_c = enumerate_candidates(view)
        old_s = pack_candidate_batch(old_c, view.topology)
        div["candidate_divergences"] += int(structural_signature(old_c) != structural_signature(bound.candidates))
        div["action_divergences"] += int(structural_signature(old_s) != structural_signature(bound.selected))
        proposal = Proposal.from_transfers(tuple(bind_action(view, local_token_ordinal=c.local_token_ordinal,
                                                             edge_index=c.edge_index, trusted_observation=obs)
                                                 for c in old_s))
        try:
            res = commit_proposal(oracle.world, obs, proposal)
            div["legal"] += int(res.legal)
            ok = True
        except (TypeError, ValueError):
            res, ok = None, False
        div["checker_divergences"] += int(ok != decision.accepted or (res is not None and (
            res.applied_actions != decision.applied_actions or res.state_version != decision.state_version)))
        div["total"] += 1
    w = oracle.world
    for o in range(state.revealed_count):
        private = w._public_to_private[state.token_ids[o]]
        div["holder_divergences"] += int(tuple(np.flatnonzero(w._possession[private])) != tuple(np.flatnonzero(state.holders[o])))
    return div


def verify_layer(layer, *, atol: float | None = None, rtol: float | None = None,
                 replay_control: bool = True) -> dict[str, Any]:
    cfg = layer.cfg
    dev = layer.device
    torch.cuda.synchronize(dev)
    from ..ops import status as _status

    _status.check(layer.status)
    W, r, T, k, S = layer.world, layer.rank, cfg.tokens_per_rank, cfg.top_k, layer.slots
    bf16 = cfg.dtype == "bf16"
    dt = torch.bfloat16 if bf16 else torch.float32
    if atol is None:
        atol = 3e-2 if bf16 else 2e-3
    if rtol is None:
        rtol = 3e-2 if bf16 else 2e-3
    epoch = int(layer.epoch.item())
    ids_t, gates_t = layer.expert_ids.clone(), layer.gates.clone()
    ids = ids_t.cpu().numpy()
    token_ids = layer.inputs.token_ids.cpu().numpy()
    off = np.asarray(cfg.chunk_offsets)
    chunk_of = np.searchsorted(off, np.arange(T), side="right") - 1
    rep: dict[str, Any] = {"epoch": epoch}

    # ---- router vs the fp32 oracle (disagreement only allowed at fp32 near-ties)
    logits = router_logits(cfg, layer.inputs.tokens, layer.weights, layer.inputs)
    chosen = logits.gather(1, ids_t.long())
    srt = torch.sort(logits, dim=-1, descending=True, stable=True)
    ref_ids = srt.indices[:, :k].to(torch.int32)
    gap_tol = 1e-4 * (1.0 + srt.values[:, :1].abs())
    mism = (ref_ids != ids_t).any(dim=1)
    near = ((srt.values[:, :k] - chosen).abs() <= gap_tol).all(dim=1)
    rep["router_mismatch"] = int((mism & ~near).sum().item())
    rep["router_near_tie_flips"] = int((mism & near).sum().item())

    # ---- oracle expert outputs for this rank's tokens (same routing)
    combined_ref, per_ref = layer_reference(cfg, layer.inputs.tokens, layer.weights, ids_t, gates_t)

    # ---- forward side: rows received by this rank
    cap = T
    rows_out = layer.rows_out.cpu().numpy()
    meta = layer._region("recv_meta", (S, W, cap, 9), torch.int64).cpu().numpy()
    seen: set[int] = set()
    fwd = {"tokens": 0, "duplicate": 0, "wrong_source": 0, "wrong_destination": 0, "wrong_expert": 0,
           "corruption": 0}
    feat = layer._region("recv_feat", (S * W * cap, cfg.hidden), dt)
    for s in range(S):
        for src in range(W):
            n = int(rows_out[s * W + src])
            if n == 0:
                continue
            m = meta[s, src, :n]
            fwd["tokens"] += n
            for key in zip(m[:, 0].tolist(), m[:, 3].tolist()):
                fwd["duplicate"] += int(key in seen)
                seen.add(key)
            fwd["wrong_source"] += int((m[:, 1] != src).sum())
            fwd["wrong_destination"] += int((m[:, 2] != r).sum())
            owners = np.array([cfg.owner(int(e), W) for e in m[:, 3]])
            slots = np.array([cfg.slot(int(e), W) for e in m[:, 3]])
            fwd["wrong_expert"] += int(((owners != r) | (slots != s)).sum())
            cs = identity_checksum_vec(m[:, :8])
            fwd["corruption"] += int((cs != m[:, 8]).sum())
            base = (s * W + src) * cap
            dig = torch.empty(n, dtype=torch.int64, device=dev)
            layer._k.feature_digest(feat[base:base + n].contiguous(), dig)
            fwd["corruption"] += int((dig.cpu().numpy() != m[:, 7]).sum())
    # ---- canary words after every array of the symmetric region
    broken = layer.guards_intact()
    rep["guards_broken"] = broken
    rep["forward"] = fwd

    # ---- return side: every (token, choice) of this rank came back exactly once
    rmeta = layer._region("ret_meta", (T * k, 8), torch.int64).cpu().numpy()
    rout = layer._region("ret_out", (T * k, cfg.out_dim), dt).float()
    ret = {"tokens": T * k, "lost": 0, "wrong_destination": 0, "wrong_return": 0, "wrong_position": 0,
           "wrong_expert": 0, "corruption": 0, "expert_output_mismatch": 0}
    tt = np.repeat(np.arange(T), k)
    ee = ids.reshape(-1).astype(np.int64)
    exp_owner = np.array([cfg.owner(int(e), W) for e in ee]) if T * k else np.zeros(0, dtype=np.int64)
    ret["lost"] = int((rmeta[:, 0] != token_ids[tt]).sum()) if T * k else 0
    ret["wrong_destination"] = int((rmeta[:, 1] != r).sum())
    ret["wrong_return"] = int((rmeta[:, 2] != exp_owner).sum())
    ret["wrong_expert"] = int((rmeta[:, 3] != ee).sum())
    ret["wrong_position"] = int(((rmeta[:, 4] != tt) | (rmeta[:, 5] != chunk_of[tt]) |
                                 (rmeta[:, 6] != tt - off[chunk_of[tt]])).sum()) if T * k else 0
    ret["corruption"] = int((identity_checksum_vec(rmeta[:, :7]) != rmeta[:, 7]).sum()) if T * k else 0
    per = per_ref.reshape(T * k, cfg.out_dim)
    close = torch.isclose(rout, per, atol=atol, rtol=rtol).all(dim=1)
    ret["expert_output_mismatch"] = int((~close).sum().item())
    rep["return"] = ret

    # ---- final output and packing counters
    out = layer.out.float()
    rep["final_combine_correct"] = bool(torch.allclose(out, combined_ref, atol=atol * max(1, k), rtol=rtol))
    rep["max_abs_err"] = float((out - combined_ref).abs().max().item()) if out.numel() else 0.0
    sc = layer.tensors["ctl_scalars"].cpu().numpy()
    rep["packing"] = {"future_access": int(sc[6]), "unrevealed_execution": int(sc[7]),
                      "duplicate_dispatch": int(sc[8]), "stale_dispatch": int(sc[9])}
    permits = layer.tensors["permit"].cpu().numpy()
    rep["permits_ok"] = bool((permits == epoch).all())
    log = layer.tensors["ctl_log"].cpu().numpy().reshape(cfg.n_desc, layer.log_stride)
    rep["guard_gate_ok"] = bool(all(int(log[d][2]) == 1 and int(log[d][7]) == 1 for d in range(cfg.n_desc)))
    if replay_control:
        rep["control"] = replay_control_fn(layer, ids, token_ids, log)
    bad = []
    for key in ("forward", "return"):
        for name, v in rep[key].items():
            if name != "tokens" and v:
                bad.append(f"{key}.{name}={v}")
    for name, v in rep["packing"].items():
        if v:
            bad.append(f"packing.{name}={v}")
    if rep["router_mismatch"]:
        bad.append(f"router_mismatch={rep['router_mismatch']}")
    if not rep["final_combine_correct"]:
        bad.append(f"final_combine max_abs_err={rep['max_abs_err']:.3g}")
    if not rep["permits_ok"] or not rep["guard_gate_ok"]:
        bad.append("control permits")
    if rep["guards_broken"]:
        bad.append(f"guard bands overwritten at offsets {rep['guards_broken']}")
    if replay_control:
        c = rep["control"]
        for name in ("device_candidate_divergences", "device_action_divergences", "candidate_divergences",
                     "action_divergences", "checker_divergences", "holder_divergences"):
            if c[name]:
                bad.append(f"control.{name}={c[name]}")
        if c["legal"] != c["total"]:
            bad.append("control.legal!=total")
    rep["pass"] = not bad
    rep["violations"] = bad
    if bad:
        raise CheckerFailure(rep)
    return rep


replay_control_fn = replay_control

__all__ = ["CheckerFailure", "OracleWorld", "control_tokens", "replay_control", "verify_layer"]

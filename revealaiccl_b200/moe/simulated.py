"""CPU "simulated ranks in one process" harness of the progressive MoE layer.

W logical ranks share a host peer memory (``HostPeerMemory``) and run the
same pipeline as the device data plane, with NumPy / PyTorch-CPU stand-ins of
the kernels:

    Router (fp32, stable top-k) -> per-trigger compiled control plane
    (StaticPlanCompiler -> IncrementalState -> FastBinder -> DynamicGuard)
    -> revealed-only packing (ProgressivePackingState) -> guarded peer
    actions (PeerCommittedAdapter) -> put / signal / receive -> forward
    verification -> expert MLP -> return payloads -> return verification ->
    gate-weighted combine at original positions.

At every trigger the compiled scheduler is compared with the uncompiled
reference planner and the trusted checker (static, single-step and
trajectory equivalence); the run also records every committed action so a
hidden-future perturbation can be checked to leave earlier triggers
unchanged.  This is the oracle of every GPU kernel and runs without a GPU.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import numpy as np
import torch

from ..scheduling.compiled import DynamicGuard, FastBinder, IncrementalState, StaticPlanCompiler, structural_signature
from ..scheduling.recourse import bind_action
from ..scheduling.robust_prefix import build_scheduling_view, enumerate_candidates, pack_candidate_batch
from ..topology.loader import load_rear4_topology
from ..transport.formats import (FORWARD_META_FIELDS, ProgressivePackingState, RouterAssignment,
                                 pack_forward_payload, pack_return_payload, verify_forward_payload,
                                 verify_return_and_combine)
from ..transport.peer_adapter import HostPeerMemory, PeerCommittedAdapter, RegisteredBufferLayout
from ..uncertainty.execution import Proposal, commit_proposal
from ..uncertainty.observation import RevealedDemandToken, TruthTokenId
from .checker import OracleWorld
from .config import MoELayerConfig
from .inputs import make_rank_inputs, make_weights
from .oracle import expert_reference, layer_reference, router_reference


@dataclass
class SimResult:
    outputs: list[torch.Tensor]
    actions: list[list[tuple[tuple[int, int], ...]]]
    counters: dict[str, int]
    equivalence: dict[str, int]
    forward_checks: list[dict] = field(default_factory=list)
    return_checks: list[dict] = field(default_factory=list)
    transport: dict[str, int] = field(default_factory=dict)


class PeerSignalMissing(RuntimeError):
    """A receiver found no ready signal for a (source, descriptor) slot."""


class SimulatedMoE:
    def __init__(self, cfg: MoELayerConfig, world: int, *, seed: int = 0, backend: str = "numpy",
                 control_topology=None) -> None:
        self.cfg, self.world, self.backend = cfg, int(world), backend
        cpu = torch.device("cpu")
        self.inputs = [make_rank_inputs(cfg, r, world, cpu, seed=seed) for r in range(world)]
        self.weights = make_weights(cfg, cpu, seed=seed)
        topo = control_topology if control_topology is not None else load_rear4_topology()[0]
        self.topology = topo
        self.plan = StaticPlanCompiler().compile(topo)
        self.route = [router_reference(cfg, inp.tokens, self.weights, inp) for inp in self.inputs]

    # ------------------------------------------------------------------ control
    def control_tokens(self, rank: int, ids: np.ndarray, chunk: int) -> list[RevealedDemandToken]:
        cfg = self.cfg
        off = cfg.chunk_offsets
        tok_ids = self.inputs[rank].token_ids.numpy()
        out = []
        for i in range(min(cfg.ctl_per_chunk, off[chunk + 1] - off[chunk])):
            pos = off[chunk] + i
            src, dst = pos % cfg.ctl_nodes, int(ids[pos, 0]) % cfg.ctl_nodes
            if src != dst:
                out.append(RevealedDemandToken(TruthTokenId(f"sim:{cfg.name}:rank{rank}:token{int(tok_ids[pos])}"),
                                               src, dst, (src,)))
        return out

    def run_control(self, rank: int, ids: np.ndarray, eq: dict[str, int]) -> tuple[list, list]:
        cfg = self.cfg
        state = IncrementalState(self.plan, max_tokens=max(1, cfg.chunks * cfg.ctl_per_chunk),
                                 max_chunks=max(8, cfg.chunks), sequence_id="", sequence_step=8)
        binder = FastBinder(self.plan, backend=self.backend)
        guard = DynamicGuard(self.plan, backend=self.backend)
        oracle = OracleWorld(self.topology, f"sim-{cfg.name}-rank{rank}")
        decisions, actions = [], []
        P, C = cfg.progressive_chunks, cfg.chunks
        for d, group in enumerate(cfg.descriptor_groups):
            toks = {c: self.control_tokens(rank, ids, c) for c in group}
            for c in group:
                state.stage_ready_chunk(c, toks[c])
            for c in group:
                state.consume_pending_chunk(c)
                oracle.append(toks[c])
            final = d >= P
            state.stage, state.ratio = (C, 1.0) if final else (d + 1, (d + 1) / C)
            bound = binder.step(state)
            dec = guard.apply(state, bound.proposal, require_scheduler_semantics=True,
                              expected_state_version=bound.state_version)
            obs = oracle.observation(stage=state.stage, ratio=state.ratio, final=final)
            view = build_scheduling_view(obs)
            old_c = enumerate_candidates(view)
            old_s = pack_candidate_batch(old_c, view.topology)
            eq["static"] += int(structural_signature(old_c) == structural_signature(bound.candidates))
            eq["single_step"] += int(structural_signature(old_s) == structural_signature(bound.selected))
            prop = Proposal.from_transfers(tuple(bind_action(view, local_token_ordinal=c.local_token_ordinal,
                                                             edge_index=c.edge_index, trusted_observation=obs)
                                                 for c in old_s))
            res = commit_proposal(oracle.world, obs, prop)
            eq["trajectory"] += int(res.legal and dec.accepted and res.applied_actions == dec.applied_actions
                                    and res.state_version == dec.state_version and prop == bound.proposal)
            eq["total"] += 1
            decisions.append(dec)
            actions.append(tuple((c.local_token_ordinal, c.edge_index) for c in bound.selected))
        eq["runtime_bfs_calls"] += binder.runtime_bfs_calls
        eq["full_rebuild_count"] += state.full_rebuild_count
        return decisions, actions

    # --------------------------------------------------------------------- run
    def run(self, arm: str = "early", routes: list | None = None, *,
            drop_signal: tuple[int, int, int] | None = None,
            corrupt_count: tuple[int, int, int] | None = None) -> SimResult:
        """One layer call over the simulated ranks.

        Host-side fault injection (each must end in a fail-closed error, never a
        silent result): ``drop_signal=(src, dst, desc)`` moves the rows of that
        action but withholds its ready signal; ``corrupt_count=(src, dst, desc)``
        rewrites the count header the receiver reads."""
        cfg, W = self.cfg, self.world
        routes = routes or self.route
        off = cfg.chunk_offsets
        D, k = cfg.hidden, cfg.top_k
        eq = {"static": 0, "single_step": 0, "trajectory": 0, "total": 0, "runtime_bfs_calls": 0,
              "full_rebuild_count": 0}
        rec_bytes = FORWARD_META_FIELDS * 8 + D * 4
        layout = RegisteredBufferLayout(W, cfg.n_desc, max(1, cfg.tokens_per_rank * k), record_bytes=rec_bytes)
        mem = HostPeerMemory(layout)
        owner = lambda e: cfg.owner(int(e), W)  # noqa: E731
        counters = {"future_access": 0, "unrevealed_execution": 0, "duplicate_dispatch": 0, "stale_dispatch": 0}
        all_actions = []
        pending: list[tuple] = []
        for r in range(W):
            ids = routes[r][0].numpy()
            decisions, acts = self.run_control(r, ids, eq)
            all_actions.append(acts)
            tok = self.inputs[r].tokens.float().numpy()
            tid = self.inputs[r].token_ids.numpy()
            words = self.inputs[r].payload_words
            packing = ProgressivePackingState(world_size=W, source_rank=r, max_chunks=cfg.chunks)
            adapter = PeerCommittedAdapter(rank=r, layout=layout)
            feats = {int(tid[t]): tok[t] for t in range(cfg.tokens_per_rank)}
            pos_of = {int(tid[t]): t for t in range(cfg.tokens_per_rank)}
            for c in range(cfg.chunks):
                assigns = [RouterAssignment(int(tid[t]), r, owner(ids[t, j]), int(ids[t, j]), c, t - off[c], int(words[t]))
                           for t in range(off[c], off[c + 1]) for j in range(k)]
                packing.mark_completed(c, assigns)
            for d, group in enumerate(cfg.descriptor_groups):
                for c in group:
                    packing.reveal(c)
                if not decisions[d].accepted:
                    raise RuntimeError("DynamicGuard rejected a descriptor")
                lay = packing.build_delta_layout(group, destination_of=owner)
                fwd = pack_forward_payload(lay, features_by_token=feats, original_position_by_token=pos_of)
                from ..transport.formats import pack_destination_layout

                shard = pack_destination_layout(lay)
                acts = adapter.commit_descriptor(shard, descriptor_id=d, guard_decision=decisions[d],
                                                 completed_chunks=range(cfg.chunks), revealed_chunks=group)
                start = 0
                for a in acts:
                    first = int(shard.offsets_tokens[a.dst_rank])
                    rows = np.concatenate([fwd.metadata[first:first + a.token_count].view(np.uint8),
                                           fwd.features[first:first + a.token_count].view(np.uint8)], axis=1) \
                        if a.token_count else np.zeros((0, rec_bytes), dtype=np.uint8)
                    mem.stage_bytes(r, a, rows)
                    if arm == "early":
                        self._put(mem, a, drop_signal, corrupt_count)
                    else:
                        pending.append(a)
                    start += a.token_count
                # local empty destination still needs a receivable (empty) slot
                if shard.sendcounts_tokens[r] == 0:
                    mem.buffers[r][layout.receive_offset(d, r):layout.receive_offset(d, r) + 8] = 0
            for name in counters:
                counters[name] += getattr(packing, {"future_access": "future_access_attempts"}.get(name, name))
        for a in pending:
            self._put(mem, a, drop_signal, corrupt_count)
        # expert ranks: receive, verify, compute, return
        fwd_checks, returns = [], {}
        for r in range(W):
            for src in range(W):
                for d in range(cfg.n_desc):
                    if src != r and not mem.wait(r, src, d):
                        # every remote (src, dst, descriptor) slot is signalled, even with zero rows
                        raise PeerSignalMissing(f"rank {r}: no ready signal from rank {src} for descriptor {d}")
                    raw = mem.receive_bytes(r, src, d)
                    if raw.shape[0] * rec_bytes > layout.peer_stride - 8:
                        raise RuntimeError(f"rank {r}: count header from rank {src} descriptor {d} exceeds its slot")
                    if raw.shape[0] == 0:
                        continue
                    meta = raw[:, :FORWARD_META_FIELDS * 8].copy().view(np.int64).reshape(-1, FORWARD_META_FIELDS)
                    feats = raw[:, FORWARD_META_FIELDS * 8:].copy().view(np.float32).reshape(-1, D)
                    chk = verify_forward_payload(meta, feats, destination_rank=r, world_size=W,
                                                 recvcounts_tokens=tuple(meta.shape[0] if s == src else 0 for s in range(W)),
                                                 destination_of=owner)
                    fwd_checks.append(chk)
                    outs = np.zeros((meta.shape[0], cfg.out_dim), dtype=np.float32)
                    for e in np.unique(meta[:, 3]):
                        sel = np.flatnonzero(meta[:, 3] == e)
                        outs[sel] = expert_reference(cfg, torch.from_numpy(feats[sel]), self.weights, int(e)).numpy()
                    ret = pack_return_payload(meta, outs, expert_rank=r, world_size=W)
                    returns.setdefault(src, []).append((r, ret))
        # source ranks: verify returns per choice slot and combine with gates
        outputs, ret_checks = [], []
        for r in range(W):
            ids, gates, _ = routes[r]
            tid = self.inputs[r].token_ids.numpy()
            combined_ref, per_ref = layer_reference(cfg, self.inputs[r].tokens, self.weights, ids, gates)
            out = torch.zeros((cfg.tokens_per_rank, cfg.out_dim))
            for j in range(k):
                metas, vals, counts = [], [], [0] * W
                for er, ret in returns.get(r, []):
                    rows = ret.metadata
                    keep = np.array([int(ids[int(m[4]), j]) == int(m[3]) for m in rows], dtype=bool)
                    metas.append(rows[keep])
                    vals.append(ret.outputs[keep])
                    counts[er] += int(keep.sum())
                meta = np.concatenate(metas) if metas else np.zeros((0, 8), np.int64)
                val = np.concatenate(vals) if vals else np.zeros((0, cfg.out_dim), np.float32)
                order = np.argsort([sum(counts[:er]) for er in range(W)], kind="stable")
                del order
                # rows must be grouped by sender in rank order for the verifier
                grouped = sorted(range(meta.shape[0]), key=lambda i: (self._sender(returns.get(r, []), meta[i]), i))
                meta, val = meta[grouped], val[grouped]
                exp_out = {int(tid[t]): (per_ref[t, j] / (gates[t, j] if float(gates[t, j]) != 0 else 1.0)).numpy()
                           for t in range(cfg.tokens_per_rank)}
                combined, chk = verify_return_and_combine(
                    meta, val, origin_rank=r, recvcounts_tokens=counts,
                    expected_expert_by_token={int(tid[t]): int(ids[t, j]) for t in range(cfg.tokens_per_rank)},
                    expected_position_by_token={int(tid[t]): t for t in range(cfg.tokens_per_rank)},
                    expected_output_by_token=exp_out, total_tokens=cfg.tokens_per_rank)
                ret_checks.append(chk)
                out += torch.from_numpy(combined) * gates[:, j:j + 1]
            outputs.append(out)
            if not torch.allclose(out, combined_ref, atol=2e-3, rtol=2e-3):
                raise RuntimeError("simulated combine does not match the oracle")
        return SimResult(outputs, all_actions, counters, eq, fwd_checks, ret_checks, dict(mem.counters))

    @staticmethod
    def _put(mem: HostPeerMemory, a, drop_signal, corrupt_count) -> None:
        key = (a.src_rank, a.dst_rank, a.descriptor_id)
        if drop_signal is not None and key == tuple(drop_signal):
            src = mem.buffers[a.src_rank][a.src_offset:a.src_offset + a.physical_bytes]
            mem.buffers[a.dst_rank][a.dst_offset:a.dst_offset + a.physical_bytes] = src  # rows, no signal
            return
        mem.put_and_signal(a)
        if corrupt_count is not None and key == tuple(corrupt_count):
            off = a.dst_offset
            bad = np.int64(a.token_count + 1)
            mem.buffers[a.dst_rank][off:off + 8] = np.frombuffer(bad.tobytes(), np.uint8)

    @staticmethod
    def _sender(returns: list, row: np.ndarray) -> int:
        return int(row[2])


__all__ = ["SimResult", "SimulatedMoE"]

"""ProgressiveMoELayer — the public entry point of the B200 data plane.

One instance per rank.  Construction (untimed set-up, like the reference's
fast data-prep precompute, rlccl/transport/fast_progressive_data_prep.py:56-67):
deterministic inputs and weights, the compiled control plan of the control
topology uploaded to the device, the symmetric peer region mapped on every
rank, per-token feature digests and linear checksum bases, and the native
runner.  ``forward(arm)`` then enqueues the whole layer without any host
synchronisation: ``arm="early"`` dispatches each descriptor right after its
scheduler trigger, ``arm="delayed"`` holds every dispatch until the final
Router chunk (the reference's C/E1 and D/D1 arms).

``verify()`` is the untimed, fail-closed post-hoc checker: forward identity
rows, return rows, expert outputs and the combined output against the fp32
oracle, the revealed-only packing counters, and a differential replay of the
device control-plane log through the compiled scheduler, the uncompiled
planner and the trusted checker.
"""

from __future__ import annotations

from dataclasses import dataclass
import math
import time
from typing import Any

import numpy as np
import torch
import torch.distributed as dist

from ..ops import status as _status
from ..ops._native import host, kernels
from ..ops.grouped_gemm import ACT_IDS, pick_bn, swiglu_interleave, swiglu_interleave_bias
from ..parallel.peer import PeerChannel, device_view
from ..scheduling.compiled import StaticPlanCompiler, _plan_flat
from ..topology.loader import load_rear4_topology
from .config import MoELayerConfig
from .inputs import make_rank_inputs, make_weights
from .oracle import layer_reference

FWD_META = 9
RET_META = 8
LOG_HEADER = 16  # 8-word decision record + 8 phase-clock words
TRACE_SLOTS = 256
GUARD_CANARY = 0x5CA1AB1E0DDC0FFE  # fills the guard band after every array of the symmetric region
PAIR_TICKET_RING = 32  # ticket slots (two words each) per GEMM CTA pair (kPairTicketRing in csrc/include/types.h)
KSPLIT_ENTRIES = 296  # GEMM-1 split-K partial tiles (two per SM); tickets as many


@dataclass
class LayerTiming:
    device_ms: float
    launches: int


class ProgressiveMoELayer:
    def __init__(self, cfg: MoELayerConfig, *, device: torch.device | str | None = None,
                 world: int | None = None, rank: int | None = None, group=None,
                 timeout_s: float = 10.0, seed: int = 0, control_topology=None,
                 control_path: str = "auto", trace: bool = False, frontend: str = "persistent",
                 gemm_pair: bool = True, pdl: bool = True, gemm_swap_max: int = 128,
                 progressive: bool = False, dispatch_ctas: int = 0, router_ring: bool = True,
                 dispatch_groups: bool = True, router_wsmem: bool = True, router_tc: bool = True,
                 gemm_ksplit: bool = True) -> None:
        self.cfg = cfg
        if world is None:
            world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        if rank is None:
            rank = dist.get_rank(group) if world > 1 else 0
        self.world, self.rank, self.group = int(world), int(rank), group
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if self.device.type != "cuda":
            raise RuntimeError("ProgressiveMoELayer runs on CUDA devices (sm_100a)")
        torch.cuda.set_device(self.device)
        self._k = kernels()
        self._h = host()
        dev = self.device
        W, T, D, E, k = self.world, cfg.tokens_per_rank, cfg.hidden, cfg.experts, cfg.top_k
        self.slots = cfg.expert_slots(W)
        bf16 = cfg.dtype == "bf16"
        dt = torch.bfloat16 if bf16 else torch.float32

        # ---- inputs and weights (deterministic)
        self.inputs = make_rank_inputs(cfg, self.rank, W, dev, seed=seed)
        self.weights = make_weights(cfg, dev, seed=seed)
        swiglu = cfg.activation == "swiglu"
        self.bn1 = pick_bn(cfg.gemm1_n, swiglu)
        self.bn2 = pick_bn(cfg.out_dim)
        F_, O = cfg.ffn_hidden, cfg.out_dim
        w1l = torch.zeros((self.slots, cfg.gemm1_n, D), dtype=dt, device=dev)
        w2l = torch.zeros((self.slots, O, F_), dtype=dt, device=dev)
        b1l = torch.zeros((self.slots, cfg.gemm1_n), dtype=torch.float32, device=dev)
        b2l = torch.zeros((self.slots, O), dtype=torch.float32, device=dev)
        self.local_experts: list[int] = []
        for s in range(self.slots):
            e = s * W + self.rank if cfg.placement == "modulo" else self.rank * self.slots + s
            if e >= E:
                self.local_experts.append(-1)
                continue
            self.local_experts.append(e)
            if swiglu:
                w1l[s] = swiglu_interleave(self.weights.w1[e:e + 1, :F_], self.weights.w1[e:e + 1, F_:], self.bn1)[0]
                if self.weights.b1 is not None:
                    b1l[s] = swiglu_interleave_bias(self.weights.b1[e:e + 1, :F_], self.weights.b1[e:e + 1, F_:], self.bn1)[0]
            else:
                w1l[s] = self.weights.w1[e]
                if self.weights.b1 is not None:
                    b1l[s] = self.weights.b1[e]
            w2l[s] = self.weights.w2[e]
            if self.weights.b2 is not None:
                b2l[s] = self.weights.b2[e]
        has_b1 = self.weights.b1 is not None
        has_b2 = self.weights.b2 is not None

        # ---- control plan (compiled once) on the device
        topo = control_topology if control_topology is not None else load_rear4_topology()[0]
        if int(topo.V) != cfg.ctl_nodes:
            raise ValueError("control topology node count must equal cfg.ctl_nodes")
        self.plan = StaticPlanCompiler().compile(topo)
        flat = _plan_flat(self.plan)
        max_tmpl = max(len(g) for g in self.plan.templates_by_destination) if self.plan.templates_by_destination else 1
        self.max_ctl_tokens = max(1, cfg.chunks * cfg.ctl_per_chunk)
        self.max_cands = max(1, self.max_ctl_tokens * max(1, max_tmpl))
        self.log_stride = LOG_HEADER + 2 * self.max_ctl_tokens + 4 * self.max_cands
        V, Ep, G = self.plan.nodes, len(self.plan.edges), len(self.plan.group_edges)
        Tc = self.max_ctl_tokens

        def dev_t(a, dtype=None):
            return torch.as_tensor(np.array(a, copy=True), device=dev, dtype=dtype)

        # ---- symmetric region shared with the peers
        ints = {
            "world": W, "rank": self.rank, "tokens": T, "hidden": D, "out_dim": O, "experts": E,
            "expert_slots": self.slots, "top_k": k, "chunks": cfg.chunks,
            "partial_chunks": cfg.progressive_chunks, "n_desc": cfg.n_desc,
            "feat_bf16": int(bf16), "out_bf16": int(bf16),
            "placement": 0 if cfg.placement == "modulo" else 1,
            "gate_mode": {"none": 0, "topk_softmax": 1, "softmax": 2}[cfg.gate_mode],
            "mask_mode": {"none": 0, "topology_source": 1}[cfg.mask_mode],
            "ctl_per_chunk": cfg.ctl_per_chunk, "ctl_nodes": cfg.ctl_nodes, "ffn": F_,
            "n1": cfg.gemm1_n, "act1": ACT_IDS[cfg.activation], "bn1": self.bn1, "bn2": self.bn2,
            "timeout_ns": int(timeout_s * 1e9), "max_cands": self.max_cands,
            "log_stride": self.log_stride, "max_ctl_tokens": Tc,
            "sms": torch.cuda.get_device_properties(dev).multi_processor_count,
            "control_serial": {"auto": 0, "serial": 1}[control_path],
            "frontend": {"steps": 0, "persistent": 1}[frontend],
            "gemm_pair": int(bool(gemm_pair)),
            "pdl": int(bool(pdl)),
            # CTA-pair GEMMs at BN = 256: a segment's last row tile of at most this
            # many rows runs with swapped operands (0 disables)
            "gemm_swap_max": int(gemm_swap_max),
            # progressive expert side: GEMM-1 CTA pairs take 256-row tiles as
            # their descriptors arrive, on the SMs of front-end workers that
            # leave after routing (dispatch_ctas workers stay to dispatch)
            "progressive": int(bool(progressive)),
            "dispatch_ctas": int(dispatch_ctas),
            # resident batches: each front-end worker streams its token groups
            # into a shared-memory ring with bulk copies ahead of routing them
            "router_ring": int(bool(router_ring)),
            # one group of front-end workers per descriptor, so released
            # descriptors are dispatched side by side (0: every worker takes a
            # share of every descriptor, one descriptor after the other)
            "dispatch_groups": int(bool(dispatch_groups)),
            # the router weights reach each worker's shared memory by one bulk
            # copy at the start of the front end (when they fit, 64 KiB)
            "router_wsmem": int(bool(router_wsmem)),
            # bf16 batches: front-end workers route 128-token units on the
            # tensor cores (tcgen05 MMA, TMA-staged tokens and weights)
            "router_tc": int(bool(router_tc)),
            # one-CTA GEMM-1 with few tiles and a long K: K split over idle SMs
            "gemm_ksplit": int(bool(gemm_ksplit)),
        }
        self.layout = self._k.sym_layout(ints)
        self.channel = PeerChannel(self.layout["total"], dev, group=group)
        if self.channel.world != W:
            raise RuntimeError("process group world size differs from the layer's world size")
        self._fill_guards()

        # ---- per-token precompute (untimed): digests and checksum bases
        self.chunk_offsets_dev = dev_t(np.asarray(cfg.chunk_offsets, dtype=np.int32))
        self.feat_digest = torch.empty(T, dtype=torch.int64, device=dev)
        self.checksum_base = torch.empty(T, dtype=torch.int64, device=dev)
        if T > 0:
            self._k.feature_digest(self.inputs.tokens, self.feat_digest)
            self._k.checksum_base(self.inputs.token_ids, self.feat_digest, self.chunk_offsets_dev,
                                  self.rank, self.checksum_base)

        rows = self.slots * W * T
        self.h = torch.empty((max(rows, 1), F_), dtype=dt, device=dev)
        self.out = torch.zeros((T, O), dtype=dt, device=dev)
        self.expert_ids = torch.zeros((T, k), dtype=torch.int32, device=dev)
        self.gates = torch.zeros((T, k), dtype=torch.float32, device=dev)
        self.status = _status.new_status(dev)
        self.epoch = torch.zeros(1, dtype=torch.int64, device=dev)
        nseg = self.slots * W
        self.segs = torch.zeros((nseg, 8), dtype=torch.int32, device=dev)
        self.rows_out = torch.zeros(nseg, dtype=torch.int32, device=dev)
        out_ptrs2 = [b + self.layout["ret_out"] for b in self.channel.bases]
        self.tensors: dict[str, Any] = {
            "tokens": self.inputs.tokens, "router_w": self.weights.router_w, "router_b": self.weights.router_b,
            "chunk_bias": self.inputs.chunk_bias, "block_mask": self.inputs.block_mask,
            "expert_ids": self.expert_ids, "gates": self.gates,
            "token_ids": self.inputs.token_ids, "feat_digest": self.feat_digest,
            "checksum_base": self.checksum_base, "chunk_offsets": self.chunk_offsets_dev,
            "sent_base": torch.zeros(E, dtype=torch.int32, device=dev),
            "desc_counts": torch.zeros(cfg.n_desc * E, dtype=torch.int32, device=dev),
            "done_counter": torch.zeros(cfg.n_desc, dtype=torch.int32, device=dev),
            "permit": torch.zeros(cfg.n_desc, dtype=torch.int64, device=dev),
            # persistent front end: chunk_done [C] + chunk_counts [C, E]; receive bases; release words
            # (+ GEMM-1 split-K tile tickets, zeroed with them every call)
            "chunk_words": torch.zeros(cfg.chunks * (1 + E) + KSPLIT_ENTRIES, dtype=torch.int32, device=dev),
            # GEMM-1 split-K partial tiles (one-CTA GEMM only: tile width < 64, no SwiGLU)
            "ksplit_partial": (torch.empty(KSPLIT_ENTRIES * 128 * self.bn1, dtype=torch.float32, device=dev)
                               if self.bn1 < 64 and cfg.activation != "swiglu" else None),
            "disp_base": torch.zeros(cfg.n_desc * E, dtype=torch.int32, device=dev),
            "desc_ready": torch.zeros(cfg.n_desc, dtype=torch.int64, device=dev),
            "epoch": self.epoch, "status": self.status,
            "bar_counter": torch.zeros(1, dtype=torch.int64, device=dev),
            # return-signal handoff: [elected epoch, parts reported, metadata CTAs done, pad]
            "ret_sync": torch.zeros(4, dtype=torch.int64, device=dev),
            # streamed inputs: per-chunk arrival words [C], resident-batch word, streamed-call flag
            "tok_ready": torch.zeros(cfg.chunks + 2, dtype=torch.int64, device=dev),
            "segs": self.segs, "rows_out": self.rows_out,
            "prefix1": torch.zeros(nseg + 1, dtype=torch.int32, device=dev),
            "prefix2": torch.zeros(nseg + 1, dtype=torch.int32, device=dev),
            "tail1": torch.zeros(nseg + 1, dtype=torch.int32, device=dev),
            "tail2": torch.zeros(nseg + 1, dtype=torch.int32, device=dev),
            "w1": w1l.reshape(self.slots * cfg.gemm1_n, D).contiguous(),
            "b1": b1l.reshape(-1).contiguous() if has_b1 else None,
            "w2": w2l.reshape(self.slots * O, F_).contiguous(),
            "b2": b2l.reshape(-1).contiguous() if has_b2 else None,
            "h": self.h, "out": self.out,
            "out_ptrs1": torch.tensor([self.h.data_ptr()] * W, dtype=torch.int64, device=dev),
            "out_ptrs2": torch.tensor(out_ptrs2, dtype=torch.int64, device=dev),
            # control plan + state: one blob (typed views below), staged by the control kernel
            "plan_E": Ep, "plan_G": G, "plan_NGM": int(flat["group_members"].size),
            "plan_NEGM": int(flat["edge_group_members"].size), "plan_NT": int(flat["tmpl_edge"].size),
            "plan_MT": int(max_tmpl),
            "ctl_blob": self._control_blob(flat, Ep, G, V, Tc, dev),
            "ctl_log": torch.zeros(cfg.n_desc * self.log_stride, dtype=torch.int32, device=dev),
            # per-peer traffic counters, updated by the dispatch and expert-plan kernels
            "peer_counters": torch.zeros(W * PeerChannel.COUNTER_STRIDE, dtype=torch.int64, device=dev),
            # progressive GEMM-1: tile list in arrival order (4 ints per tile), its
            # published length, the per-call ticket counter and each CTA pair's ticket ring
            "tile_list": torch.zeros(4 * self._max_tiles1(nseg), dtype=torch.int32, device=dev),
            "tile_word": torch.zeros(1, dtype=torch.int64, device=dev),
            "ticket_counter": torch.zeros(1, dtype=torch.int32, device=dev),
            "pair_tickets": torch.zeros((ints["sms"] // 2) * PAIR_TICKET_RING * 2, dtype=torch.int64, device=dev),
        }
        self.tensors = {kk: v for kk, v in self.tensors.items() if v is not None}
        self.channel.bind_counters(self.tensors["peer_counters"])
        self.tensors.update(self._ctl_views)
        if trace:  # device trace ring: 32-byte slots, one per launch of a call
            self.tensors["trace"] = torch.zeros(TRACE_SLOTS * 4, dtype=torch.int64, device=dev)
        self.router_stream = torch.cuda.Stream(device=dev)
        self.comm_stream = torch.cuda.Stream(device=dev)
        self.copy_stream = torch.cuda.Stream(device=dev)  # streamed token chunks (H2D)
        torch.cuda.synchronize(dev)
        self.runner = self._k.MoELayerRunner(
            ints, self.tensors, [int(b) for b in self.channel.bases], list(cfg.chunk_offsets),
            self.router_stream.cuda_stream, self.comm_stream.cuda_stream)
        self._graph_arm: str | None = None
        self.launches_per_call = 0
        if W > 1:
            dist.barrier(group=group)

    def _max_tiles1(self, nseg: int) -> int:
        """Upper bound of GEMM-1's 256-row tiles: every row this rank can
        receive (all ranks' tokens x top-k) plus one partial tile per
        segment, times the column blocks."""
        cfg = self.cfg
        rows = self.world * cfg.tokens_per_rank * cfg.top_k
        return (rows // 256 + nseg + 1) * max(1, cfg.gemm1_n // self.bn1)

    def _control_blob(self, flat, Ep: int, G: int, V: int, Tc: int, dev) -> torch.Tensor:
        """One device buffer holding the compiled plan, the scheduler state, the
        trigger scalars and scratch at the offsets of the native layout; the
        plan part is filled here, the rest is (re)initialised by the kernel."""
        cfg = self.cfg
        if cfg.chunks > 64:
            raise ValueError("the device control plane tracks at most 64 chunks (64-bit chunk bitmaps)")
        lay = self._k.control_layout({
            "E": Ep, "G": G, "V": V, "T": Tc, "n_gm": int(flat["group_members"].size),
            "n_egm": int(flat["edge_group_members"].size), "n_tmpl": int(flat["tmpl_edge"].size),
            "max_cands": self.max_cands, "chunks": cfg.chunks})
        blob = torch.zeros(int(lay["total"]), dtype=torch.uint8, device=dev)
        dtypes = {1: torch.uint8, 4: torch.int32, 8: torch.int64}
        views = {}
        for name, (off, count, elem) in lay["arrays"].items():
            n = max(int(count), 1)
            views[name] = blob[int(off):int(off) + n * int(elem)].view(dtypes[int(elem)])
        for name in ("edge_src", "edge_tgt", "cap_units", "group_limits", "group_ptr", "group_members",
                     "edge_group_ptr", "edge_group_members", "distances", "tmpl_ptr", "tmpl_edge", "tmpl_src",
                     "tmpl_tgt", "tmpl_tdist"):
            a = np.asarray(flat[name]).reshape(-1)
            if a.size:
                views[name][: a.size].copy_(torch.as_tensor(a.astype(np.int64 if views[name].dtype == torch.int64
                                                                    else np.int32)))
        self.control_layout = lay
        self._ctl_views = views
        return blob

    # ------------------------------------------------------------------ run
    def forward(self, arm: str = "early") -> torch.Tensor:
        """Enqueue one layer call on the layer's comm stream (no host sync)."""
        if arm not in ("early", "delayed"):
            raise ValueError("arm must be 'early' or 'delayed'")
        self.comm_stream.wait_stream(torch.cuda.current_stream(self.device))
        self.launches_per_call = self.runner.forward(arm == "delayed")
        torch.cuda.current_stream(self.device).wait_stream(self.comm_stream)
        return self.out

    def capture(self, arm: str = "early") -> int:
        """Record one layer call of ``arm`` as a CUDA graph (call ``forward`` once before)."""
        torch.cuda.synchronize(self.device)
        n = self.runner.capture(arm == "delayed")
        self._graph_arm = arm
        self.launches_per_call = n
        return n

    def replay(self, arm: str | None = None) -> torch.Tensor:
        """Relaunch the captured graph of ``arm`` (default: the last captured arm)."""
        arm = arm or self._graph_arm or "early"
        self.comm_stream.wait_stream(torch.cuda.current_stream(self.device))
        self.launches_per_call = self.runner.replay(arm == "delayed")
        torch.cuda.current_stream(self.device).wait_stream(self.comm_stream)
        return self.out

    def device_barrier(self) -> None:
        """Align every rank on the device (cross-GPU flag barrier on the comm stream)."""
        self.comm_stream.wait_stream(torch.cuda.current_stream(self.device))
        self.runner.device_barrier()

    def load_tokens_(self, host_tokens: torch.Tensor) -> None:
        """Copy a new [T, D] token batch from (pinned) host memory on the comm
        stream and refresh its per-token digests and checksum bases."""
        with torch.cuda.stream(self.comm_stream):
            self.inputs.tokens.copy_(host_tokens, non_blocking=True)
            if self.cfg.tokens_per_rank:
                self._k.feature_digest(self.inputs.tokens, self.feat_digest)
                self._k.checksum_base(self.inputs.token_ids, self.feat_digest, self.chunk_offsets_dev,
                                      self.rank, self.checksum_base)

    def __call__(self, host_tokens: torch.Tensor, host_out: torch.Tensor | None = None,
                 arm: str = "early") -> torch.Tensor:
        """End-to-end call: pinned host tokens in, combined output back in host
        memory (the captured graph of ``arm`` is used when one exists).

        With the persistent front end the batch is streamed: each router
        chunk's rows are copied on the copy stream and published to the
        running front end, whose workers route a chunk as soon as it lands and
        digest its rows on the way, so the host-to-device copy of later chunks
        overlaps the routing, control and dispatch of earlier ones."""
        cur = torch.cuda.current_stream(self.device)
        streamed = (self.runner.persistent_frontend() and host_tokens.is_pinned() and host_tokens.is_contiguous()
                    and host_tokens.dtype == self.inputs.tokens.dtype and host_tokens.shape == self.inputs.tokens.shape)
        if streamed:
            self.copy_stream.wait_stream(cur)
            self.comm_stream.wait_stream(cur)
            # copies and stream writes only: no kernels beyond the layer's own
            self.launches_per_call = self.runner.stream_call(host_tokens.data_ptr(), self.copy_stream.cuda_stream,
                                                             arm == "delayed")
        else:
            self.load_tokens_(host_tokens)
            if self.runner.has_graph(arm == "delayed"):
                self.launches_per_call = self.runner.replay(arm == "delayed") + 2
            else:
                self.launches_per_call = self.runner.forward(arm == "delayed") + 2
        if host_out is None:
            host_out = torch.empty(self.out.shape, dtype=self.out.dtype, pin_memory=True)
        with torch.cuda.stream(self.comm_stream):
            host_out.copy_(self.out, non_blocking=True)
        torch.cuda.current_stream(self.device).wait_stream(self.comm_stream)
        return host_out

    def clear_returns(self) -> None:
        """Zero this rank's return rows and return identity rows (so a lost
        return row cannot hide behind a previous call's row); collective-free,
        call between layer calls.  The guard bands stay as they are."""
        torch.cuda.synchronize(self.device)
        guards = self.layout["guards"]
        for name, guard in (("ret_out", guards[6]), ("ret_meta", guards[7])):
            self._region(name, (guard - self.layout[name],), torch.uint8).zero_()
        torch.cuda.synchronize(self.device)

    def _fill_guards(self) -> None:
        """Write the canary pattern into every guard band of this rank's region."""
        n = int(self.layout["guard_bytes"]) // 8
        for off in self.layout["guards"]:
            self.channel.view(int(off), (n,), torch.int64).fill_(GUARD_CANARY)
        torch.cuda.synchronize(self.device)

    def guards_intact(self) -> list[int]:
        """Offsets of this rank's guard bands whose canary changed (empty: all intact)."""
        torch.cuda.synchronize(self.device)
        n = int(self.layout["guard_bytes"]) // 8
        return [int(off) for off in self.layout["guards"]
                if not bool((self.channel.view(int(off), (n,), torch.int64) == GUARD_CANARY).all().item())]

    def wait(self) -> None:
        torch.cuda.current_stream(self.device).wait_stream(self.comm_stream)

    def trace_events(self) -> list[dict[str, Any]]:
        """Device spans of the launches of the last layer call (layer built with
        ``trace=True``): kernel kind, its argument (chunk / descriptor / -1),
        %globaltimer start and end in ns, and the number of CTAs that ran."""
        if "trace" not in self.tensors:
            raise RuntimeError("layer was built without trace=True")
        torch.cuda.synchronize(self.device)
        raw = self.tensors["trace"].view(-1, 4).cpu()
        out = []
        for i, (kind, arg) in enumerate(self.runner.trace_labels()):
            start, end, meta = (int(raw[i, 0]) & (2**64 - 1)), int(raw[i, 1]), int(raw[i, 2])
            ctas = meta & 0xFFFFFFFF
            if ctas == 0:
                continue  # the launch did not run (or ran no CTA)
            out.append({"kind": kind, "arg": int(arg), "start_ns": start, "end_ns": end, "ctas": ctas,
                        "rank": self.rank})
        return out

    def inject_skip_signal(self, desc: int = -1) -> None:
        """Host-side fault injection for failure-detection tests: descriptor
        ``desc``'s dispatch withholds its ready flags (receivers time out after
        ``timeout_s`` and record a status); -1 turns it off.  Applies to the
        next ``forward`` (re-``capture`` a graph to include it)."""
        self.runner.inject_skip_signal(int(desc))

    def clear_status(self) -> None:
        """Zero the device status record (after a reported failure)."""
        self.status.zero_()
        torch.cuda.synchronize(self.device)

    def status_record(self) -> dict:
        torch.cuda.synchronize(self.device)
        return _status.decode(self.status)

    def check_status(self) -> None:
        torch.cuda.synchronize(self.device)
        _status.check(self.status)

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        self.runner = None
        self.channel.close()

    # --------------------------------------------------------------- checker
    def _region(self, name: str, shape, dtype, rank: int | None = None) -> torch.Tensor:
        return self.channel.view(self.layout[name], shape, dtype, rank)

    def verify(self, *, atol: float | None = None, rtol: float | None = None,
               replay_control: bool = True) -> dict[str, Any]:
        """Fail-closed post-hoc checker of the last layer call (collective: every
        rank must call it; it raises on any violation)."""
        from .checker import verify_layer

        return verify_layer(self, atol=atol, rtol=rtol, replay_control=replay_control)


__all__ = ["LayerTiming", "ProgressiveMoELayer"]

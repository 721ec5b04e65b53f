"""Lower a slot schedule to an MSCCL XML program, and check the program.

A schedule is a list of per-slot 0/1 matrices ``Y_t[c, e]`` (chunk ``c``
crosses edge ``e`` in slot ``t``).  The reference converts one through
MSCCLang (rlccl/utils/xml_converter.py, which needs msccl-tools); this module
writes the XML itself, in four stages:

1. ``gpu_transfers`` — GPU-to-GPU transfers per slot.  Non-GPU vertices
   (switches, NICs) keep no buffer: a chunk delivered to one at slot t-1 can
   be forwarded only at slot t.  Every switch -> GPU delivery is traced back
   hop by hop (one slot per hop) to the GPU that injected the chunk, and the
   transfer is placed at that GPU's send slot.  The whole schedule is
   validated on the way (a source must hold the chunk at the start of its
   slot; a GPU holds a chunk from the slot it arrives in).
2. Collective layout — AllGather: rank r's i-th input chunk lands at output
   index r * chunk_factor + i everywhere; AllToAll: the j-th chunk from rank s
   to rank d sits at input[s][d * cf + j] and lands at output[d][s * cf + j].
3. Program — a list of copies (round, source rank/buffer/index, destination
   rank/buffer/index).  AllGather copies each chunk into its own output slot,
   then follows the schedule's transfers output to output.  AllToAll follows
   each chunk's GPU path, relaying through scratch slots of intermediate
   GPUs, or copies it straight across when the schedule moves it in one hop.
4. XML — each rank gets threadblocks per (send peer, receive peer, channel);
   a cross-rank copy is a send step on the source and a receive step on the
   destination, a local one a copy step; a step that reads a slot another
   threadblock wrote depends on that step (``depid``/``deps``, ``hasdep`` on
   the writer).  ``instances`` replicates the program on that many channels,
   each moving one slice of every chunk; ``instr_fusion`` fuses a receive
   whose only reader is a send into one receive-copy-send step.

``check_xml`` executes a program on the XML alone — per-channel FIFO links,
dependencies, threadblock order — and verifies the collective's
postcondition, reporting a deadlock or a wrong slot.
"""

from __future__ import annotations

import argparse
from collections import defaultdict, deque
from dataclasses import dataclass
from typing import Sequence
import xml.etree.ElementTree as ET
from xml.sax.saxutils import quoteattr

import numpy as np

COLLECTIVES = ("allgather", "alltoall")


# ------------------------------------------------------------------ stage 1
def gpu_transfers(schedule: Sequence[np.ndarray], edge_src: np.ndarray, edge_dst: np.ndarray,
                  pre: np.ndarray, is_switch: np.ndarray,
                  chunk_mask: np.ndarray | None = None) -> list[list[tuple[int, int, int]]]:
    """Per slot, the (source GPU, destination GPU, chunk) transfers of a schedule."""
    src, dst = np.asarray(edge_src, dtype=np.int64), np.asarray(edge_dst, dtype=np.int64)
    pre = np.asarray(pre) > 0
    sw = np.asarray(is_switch, dtype=bool)
    C, V = pre.shape
    valid = np.ones(C, dtype=bool) if chunk_mask is None else np.asarray(chunk_mask, dtype=bool).reshape(C)
    sent = []
    for t, Y in enumerate(schedule):
        Y = np.asarray(Y)
        if Y.ndim == 3:
            if Y.shape[0] != 1:
                raise ValueError(f"slot {t}: one schedule instance expected")
            Y = Y[0]
        if Y.shape != (C, len(src)):
            raise ValueError(f"slot {t}: schedule shape {Y.shape} != ({C}, {len(src)})")
        sent.append((Y > 0) & valid[:, None])
    # forward pass: GPUs keep what they hold; a switch holds only last slot's deliveries
    held = pre & ~sw[None, :] & valid[:, None]
    inbox = np.zeros_like(held)
    for t, S in enumerate(sent):
        have = held | inbox
        c_idx, e_idx = np.nonzero(S)
        bad = ~have[c_idx, src[e_idx]]
        if bad.any():
            i = int(np.flatnonzero(bad)[0])
            raise ValueError(f"slot {t}: chunk {c_idx[i]} is not at vertex {src[e_idx[i]]} for edge {e_idx[i]}")
        got = np.zeros_like(held)
        got[c_idx, dst[e_idx]] = True
        held |= got & ~sw[None, :]
        inbox = got & sw[None, :]
    into: list[list[int]] = [[] for _ in range(V)]
    for e in range(len(src)):
        into[int(dst[e])].append(e)

    def injector(t: int, c: int, node: int) -> tuple[int, int]:
        while sw[node]:
            if t == 0:
                raise ValueError(f"switch {node} forwards chunk {c} at slot 0")
            feed = [e for e in into[node] if sent[t - 1][c, e]]
            if not feed:
                raise ValueError(f"switch {node} forwards chunk {c} at slot {t} that nothing delivered at {t - 1}")
            node, t = int(src[feed[0]]), t - 1
        return node, t

    rounds: list[list[tuple[int, int, int]]] = [[] for _ in sent]
    arrivals: list[list[tuple[int, int]]] = [[] for _ in sent]
    for t, S in enumerate(sent):
        for c, e in zip(*np.nonzero(S)):
            u, v = int(src[e]), int(dst[e])
            if sw[v]:
                continue
            g, ts = injector(t, int(c), u)
            rounds[ts].append((g, v, int(c)))
            arrivals[t].append((v, int(c)))
    holders = [set(np.flatnonzero(held_row).tolist()) for held_row in (pre & ~sw[None, :] & valid[:, None])]
    for t in range(len(sent)):
        for g, _, c in rounds[t]:
            if g not in holders[c]:
                raise ValueError(f"slot {t}: GPU {g} sends chunk {c} before holding it")
        for v, c in arrivals[t]:
            holders[c].add(v)
    return rounds


# ------------------------------------------------------------------ stage 2
@dataclass(frozen=True)
class Placement:
    chunk_id: int
    origin_rank: int
    origin_index: int
    dest_rank: int       # AllGather: -1 (every rank)
    dest_index: int      # AllGather: the global output index


def _ranks(is_switch: np.ndarray) -> tuple[list[int], dict[int, int]]:
    gpus = [int(v) for v in np.flatnonzero(~np.asarray(is_switch, dtype=bool))]
    if not gpus:
        raise ValueError("the topology has no GPU vertex")
    return gpus, {v: r for r, v in enumerate(gpus)}


def _single_gpu(row: np.ndarray, is_switch: np.ndarray, what: str, c: int) -> int:
    vs = [int(v) for v in np.flatnonzero(np.asarray(row) > 0) if not is_switch[v]]
    if len(vs) != 1:
        raise ValueError(f"chunk {c}: expected exactly one GPU {what}, got {vs}")
    return vs[0]


def allgather_layout(pre: np.ndarray, is_switch: np.ndarray, chunk_mask=None) -> tuple[list[Placement], int]:
    pre = np.asarray(pre)
    sw = np.asarray(is_switch, dtype=bool)
    _, v2r = _ranks(sw)
    C = pre.shape[0]
    valid = np.ones(C, dtype=bool) if chunk_mask is None else np.asarray(chunk_mask, dtype=bool).reshape(C)
    per_rank: dict[int, list[int]] = defaultdict(list)
    for c in np.flatnonzero(valid).tolist():
        per_rank[v2r[_single_gpu(pre[c], sw, "owner", c)]].append(c)
    if not per_rank:
        raise ValueError("no valid chunk")
    cf = max(len(v) for v in per_rank.values())
    if any(len(v) != cf for v in per_rank.values()):
        raise ValueError(f"AllGather needs the same chunk count on every rank that owns chunks: "
                         f"{ {r: len(v) for r, v in per_rank.items()} }")
    out = [Placement(c, r, i, -1, r * cf + i) for r, cs in per_rank.items() for i, c in enumerate(sorted(cs))]
    return sorted(out, key=lambda p: p.chunk_id), cf


def alltoall_layout(pre: np.ndarray, post: np.ndarray, is_switch: np.ndarray,
                    chunk_mask=None) -> tuple[list[Placement], int]:
    pre, post = np.asarray(pre), np.asarray(post)
    sw = np.asarray(is_switch, dtype=bool)
    _, v2r = _ranks(sw)
    C = pre.shape[0]
    valid = np.ones(C, dtype=bool) if chunk_mask is None else np.asarray(chunk_mask, dtype=bool).reshape(C)
    pairs: dict[tuple[int, int], list[int]] = defaultdict(list)
    for c in np.flatnonzero(valid).tolist():
        s = v2r[_single_gpu(pre[c], sw, "source", c)]
        d = v2r[_single_gpu(post[c], sw, "destination", c)]
        pairs[(s, d)].append(c)
    if not pairs:
        raise ValueError("no valid chunk")
    cf = max(len(v) for v in pairs.values())
    out = [Placement(c, s, d * cf + j, d, s * cf + j) for (s, d), cs in pairs.items() for j, c in enumerate(sorted(cs))]
    return sorted(out, key=lambda p: p.chunk_id), cf


# ------------------------------------------------------------------ stage 3
@dataclass(frozen=True)
class Copy:
    round: int
    src_rank: int
    src_buf: str   # "i", "o" or "s"
    src_idx: int
    dst_rank: int
    dst_buf: str
    dst_idx: int


def allgather_program(rounds, placements: list[Placement], v2r: dict[int, int]) -> list[Copy]:
    glob = {p.chunk_id: p.dest_index for p in placements}
    prog = [Copy(-1, p.origin_rank, "i", p.origin_index, p.origin_rank, "o", p.dest_index) for p in placements]
    for t, tr in enumerate(rounds):
        for u, v, c in tr:
            if c in glob and v2r[u] != v2r[v]:
                prog.append(Copy(t, v2r[u], "o", glob[c], v2r[v], "o", glob[c]))
    return prog


def alltoall_program(rounds, placements: list[Placement], v2r: dict[int, int]) -> tuple[list[Copy], int]:
    """Copies along each chunk's GPU path; returns (program, scratch slots per rank)."""
    hops: dict[int, list[tuple[int, int, int]]] = defaultdict(list)
    for t, tr in enumerate(rounds):
        for u, v, c in tr:
            hops[c].append((t, v2r[u], v2r[v]))
    scratch_next: dict[int, int] = defaultdict(int)
    prog: list[Copy] = []
    for p in placements:
        path = _chain(hops.get(p.chunk_id, []), p.origin_rank, p.dest_rank)
        if p.origin_rank == p.dest_rank or not path:
            prog.append(Copy(path[-1][0] if path else -1, p.origin_rank, "i", p.origin_index, p.dest_rank, "o",
                             p.dest_index))
            continue
        buf, idx = "i", p.origin_index
        for k, (t, u, v) in enumerate(path):
            if k == len(path) - 1:
                prog.append(Copy(t, u, buf, idx, v, "o", p.dest_index))
            else:
                slot = scratch_next[v]
                scratch_next[v] += 1
                prog.append(Copy(t, u, buf, idx, v, "s", slot))
                buf, idx = "s", slot
    prog.sort(key=lambda cp: cp.round)
    return prog, max(scratch_next.values(), default=0)


def _chain(hops, origin: int, dest: int) -> list[tuple[int, int, int]]:
    """The first time-ordered hop sequence origin -> dest among a chunk's hops."""
    at, path, t_min = origin, [], -1
    for t, u, v in sorted(hops):
        if u == at and t > t_min:
            path.append((t, u, v))
            at, t_min = v, t
            if at == dest:
                return path
    return []


# ------------------------------------------------------------------ stage 4
def _fusion_candidates(program: list[Copy]) -> dict[int, int]:
    """Forward copies j whose source slot was landed by a cross-rank copy i and
    has no other reader: {j: i}."""
    cross = [(j, cp) for j, cp in enumerate(program) if cp.src_rank != cp.dst_rank]
    landed = {(cp.dst_rank, cp.dst_buf, cp.dst_idx): j for j, cp in cross}
    reads: dict[tuple[int, str, int], int] = defaultdict(int)
    for cp in program:
        reads[(cp.src_rank, cp.src_buf, cp.src_idx)] += 1
    out: dict[int, int] = {}
    for j, cp in cross:
        key = (cp.src_rank, cp.src_buf, cp.src_idx)
        i = landed.get(key)
        if i is not None and reads[key] == 1 and program[i].round <= cp.round:
            out[j] = i
    return out


def _send_key(program: list[Copy], fuse: dict[int, int], k: int) -> tuple[int, int, int]:
    """Position of copy k's send among its threadblock's steps: a fused send
    goes out with the receive it is fused to."""
    i = fuse.get(k)
    return (program[i].round, 1, i) if i is not None else (program[k].round, 0, k)


def _link_order_kept(program: list[Copy], fuse: dict[int, int], r: int, b: int) -> bool:
    """Rank r issues its sends to b in the order b lists its receives from r."""
    sends = [k for k, cp in enumerate(program) if cp.src_rank == r and cp.dst_rank == b]
    return (sorted(sends, key=lambda k: _send_key(program, fuse, k))
            == sorted(sends, key=lambda k: (program[k].round, 1, k)))


def lower_to_xml(program: list[Copy], *, ngpus: int, in_chunks: int, out_chunks: int, scratch_chunks: int,
                 coll: str, name: str, instances: int = 1, instr_fusion: bool = False,
                 proto: str = "Simple") -> str:
    """MSCCL XML of a copy program (see the module notes for the lowering rules)."""
    if instances < 1:
        raise ValueError("instances >= 1")
    candidates = _fusion_candidates(program) if instr_fusion else {}
    # threadblock peers per rank: a receive peer and a send peer share a
    # threadblock when fused steps need both (most candidates first), every
    # other peer gets its own
    votes: dict[int, dict[tuple[int, int], int]] = defaultdict(lambda: defaultdict(int))
    for j, i in candidates.items():
        votes[program[j].src_rank][(program[i].src_rank, program[j].dst_rank)] += 1
    send_pair: dict[tuple[int, int], int] = {}  # (rank, send peer) -> paired recv peer
    recv_pair: dict[tuple[int, int], int] = {}
    for r, vs in votes.items():
        for (a, b), _ in sorted(vs.items(), key=lambda kv: (-kv[1], kv[0])):
            if (r, b) not in send_pair and (r, a) not in recv_pair:
                send_pair[(r, b)], recv_pair[(r, a)] = a, b
    # a fusion keeps the receive where it was and moves the send up to it; it
    # is taken only if the relay's sends on that link keep the receiver's order
    fuse: dict[int, int] = {}
    for j, i in sorted(candidates.items()):
        r, b = program[j].src_rank, program[j].dst_rank
        if send_pair.get((r, b)) == program[i].src_rank and _link_order_kept(program, {**fuse, j: i}, r, b):
            fuse[j] = i
    absorbed = set(fuse.values())

    def send_tb(r, b):
        return (r, b, send_pair.get((r, b), -1))

    def recv_tb(r, a):
        return (r, recv_pair.get((r, a), -1), a)

    # steps per (rank, send, recv) on one channel; order key (round, phase):
    # sends of a round go before its receives (a send never needs a slot the
    # same round fills), so no two threadblocks wait on each other's receive
    steps: dict[tuple[int, int, int], list[tuple[tuple[int, int, int], dict]]] = defaultdict(list)
    for j, cp in enumerate(program):
        src, dst = (cp.src_buf, cp.src_idx), (cp.dst_buf, cp.dst_idx)
        if cp.src_rank == cp.dst_rank:
            steps[(cp.src_rank, -1, -1)].append(((cp.round, 1, j), dict(type="cpy", src=src, dst=dst, writes=dst)))
            continue
        if j in fuse:
            prev = program[fuse[j]]
            land = (prev.dst_buf, prev.dst_idx)
            steps[send_tb(cp.src_rank, cp.dst_rank)].append(
                ((prev.round, 1, fuse[j]), dict(type="rcs", src=land, dst=dst, writes=land)))
        else:
            steps[send_tb(cp.src_rank, cp.dst_rank)].append(((cp.round, 0, j), dict(type="s", src=src, dst=dst)))
        if j not in absorbed:
            steps[recv_tb(cp.dst_rank, cp.src_rank)].append(((cp.round, 1, j), dict(type="r", src=dst, dst=dst,
                                                                                     writes=dst)))
    for key in steps:
        steps[key].sort(key=lambda kv: kv[0])
    keys = sorted(steps)
    per_rank_ids: dict[int, int] = defaultdict(int)
    tb_index: dict[tuple[int, tuple[int, int, int]], int] = {}
    for inst in range(instances):
        for key in keys:
            tb_index[(inst, key)] = per_rank_ids[key[0]]
            per_rank_ids[key[0]] += 1
    writer: dict[tuple[int, int, str, int], tuple[int, int]] = {}
    for inst in range(instances):
        for key in keys:
            for s_i, (_, st) in enumerate(steps[key]):
                if "writes" in st:
                    writer[(inst, key[0]) + st["writes"]] = (tb_index[(inst, key)], s_i)
    needed: set[tuple[int, int, int]] = set()
    deps: dict[tuple[int, tuple[int, int, int], int], tuple[int, int]] = {}
    for inst in range(instances):
        for key in keys:
            for s_i, (_, st) in enumerate(steps[key]):
                if st["type"] in ("s", "cpy"):
                    w = writer.get((inst, key[0]) + st["src"])
                    if w is not None and w[0] != tb_index[(inst, key)]:
                        deps[(inst, key, s_i)] = w
                        needed.add((key[0],) + w)
    lines = [f'<algo name={quoteattr(name)} proto="{proto}" nchannels="{instances}" '
             f'nchunksperloop="{out_chunks * instances}" ngpus="{ngpus}" coll="{coll}" inplace="0">']
    for g in range(ngpus):
        lines.append(f'  <gpu id="{g}" i_chunks="{in_chunks * instances}" o_chunks="{out_chunks * instances}" '
                     f's_chunks="{scratch_chunks * instances}">')
        for inst in range(instances):
            for key in (k for k in keys if k[0] == g):
                tid = tb_index[(inst, key)]
                lines.append(f'    <tb id="{tid}" send="{key[1]}" recv="{key[2]}" chan="{inst}">')
                for s_i, (_, st) in enumerate(steps[key]):
                    (sb, so), (db, do) = st["src"], st["dst"]
                    dep = deps.get((inst, key, s_i), (-1, -1))
                    lines.append(f'      <step s="{s_i}" type="{st["type"]}" srcbuf="{sb}" '
                                 f'srcoff="{so * instances + inst}" dstbuf="{db}" dstoff="{do * instances + inst}" '
                                 f'cnt="1" depid="{dep[0]}" deps="{dep[1]}" hasdep="{int((g, tid, s_i) in needed)}"/>')
                lines.append("    </tb>")
        lines.append("  </gpu>")
    lines.append("</algo>")
    return "\n".join(lines) + "\n"


# ------------------------------------------------------------------- check
def check_xml(xml: str, expect_output, initial_input) -> dict:
    """Run the program on its XML alone and compare every output slot.

    initial_input(rank, index) -> token in input slot; expect_output(rank,
    index) -> token that must end in output slot (None: unconstrained).
    Raises ValueError on a deadlock, a receive of the wrong slot or a wrong
    output; returns counts of executed steps."""
    root = ET.fromstring(xml)
    inst = int(root.get("nchannels", "1"))
    bufs: dict[tuple[int, str], dict[int, object]] = defaultdict(dict)
    progs = []
    for gpu in root.iter("gpu"):
        g = int(gpu.get("id"))
        for i in range(int(gpu.get("i_chunks"))):
            bufs[(g, "i")][i] = initial_input(g, i // inst, i % inst)
        for tb in gpu.iter("tb"):
            steps = [dict(s.attrib) for s in tb.iter("step")]
            progs.append({"g": g, "id": int(tb.get("id")), "send": int(tb.get("send")), "recv": int(tb.get("recv")),
                          "chan": int(tb.get("chan")), "steps": steps, "pc": 0})
    done: set[tuple[int, int, int]] = set()
    links: dict[tuple[int, int, int], deque] = defaultdict(deque)
    executed = 0
    while True:
        moved = False
        for tb in progs:
            while tb["pc"] < len(tb["steps"]):
                st = tb["steps"][tb["pc"]]
                dep = (tb["g"], int(st["depid"]), int(st["deps"]))
                if dep[1] >= 0 and dep not in done:
                    break
                kind = st["type"]
                src = (tb["g"], st["srcbuf"]), int(st["srcoff"])
                dst = (tb["g"], st["dstbuf"]), int(st["dstoff"])
                if kind in ("r", "rcs"):
                    q = links[(tb["recv"], tb["g"], tb["chan"])]
                    if not q:
                        break
                    token, to_slot = q.popleft()
                    land = dst if kind == "r" else src
                    if to_slot != (land[0][1], land[1]):
                        raise ValueError(f"gpu {tb['g']} tb {tb['id']}: received slot {to_slot}, expected {land}")
                    bufs[land[0]][land[1]] = token
                    if kind == "rcs":
                        links[(tb["g"], tb["send"], tb["chan"])].append((token, (st["dstbuf"], int(st["dstoff"]))))
                elif kind == "s":
                    if src[1] not in bufs[src[0]]:
                        raise ValueError(f"gpu {tb['g']} sends empty slot {src}")
                    links[(tb["g"], tb["send"], tb["chan"])].append((bufs[src[0]][src[1]], (dst[0][1], dst[1])))
                elif kind == "cpy":
                    bufs[dst[0]][dst[1]] = bufs[src[0]][src[1]]
                else:
                    raise ValueError(f"unknown step type {kind}")
                done.add((tb["g"], tb["id"], tb["pc"]))
                tb["pc"] += 1
                executed += 1
                moved = True
        if not moved:
            break
    stuck = [(tb["g"], tb["id"], tb["pc"]) for tb in progs if tb["pc"] < len(tb["steps"])]
    if stuck:
        raise ValueError(f"the program deadlocks at (gpu, tb, step) {stuck[:4]}")
    wrong = 0
    for gpu in root.iter("gpu"):
        g = int(gpu.get("id"))
        for i in range(int(gpu.get("o_chunks"))):
            want = expect_output(g, i // inst, i % inst)
            if want is not None and bufs[(g, "o")].get(i) != want:
                wrong += 1
    if wrong:
        raise ValueError(f"{wrong} output slots hold the wrong chunk")
    return {"steps": executed, "threadblocks": len(progs)}


# -------------------------------------------------------------------- glue
def schedule_to_msccl_xml(schedule: Sequence[np.ndarray], *, edge_src, edge_dst, pre_condition,
                          post_condition=None, is_switch=None, chunk_mask=None, collective: str = "allgather",
                          name: str = "raiccl_schedule", instances: int = 1, instr_fusion: bool = False,
                          check: bool = True) -> str:
    """The whole lowering: schedule -> GPU transfers -> collective program -> XML (checked)."""
    pre = np.asarray(pre_condition)
    pre = pre[0] if pre.ndim == 3 else pre
    V = pre.shape[1]
    sw = np.zeros(V, dtype=bool) if is_switch is None else np.asarray(is_switch, dtype=bool).reshape(V)
    mask = None if chunk_mask is None else np.asarray(chunk_mask).reshape(-1)
    rounds = gpu_transfers(schedule, edge_src, edge_dst, pre, sw, mask)
    gpus, v2r = _ranks(sw)
    n = len(gpus)
    coll = collective.lower()
    if coll == "allgather":
        places, cf = allgather_layout(pre, sw, mask)
        prog = allgather_program(rounds, places, v2r)
        xml = lower_to_xml(prog, ngpus=n, in_chunks=cf, out_chunks=n * cf, scratch_chunks=0, coll="allgather",
                           name=name, instances=instances, instr_fusion=instr_fusion)
        if check:
            live = {p.dest_index for p in places}
            check_xml(xml, lambda r, i, k: ("c", i, k) if i in live else None,
                      lambda r, i, k: ("c", r * cf + i, k))
    elif coll == "alltoall":
        if post_condition is None:
            raise ValueError("AllToAll needs the post-condition (each chunk's destination)")
        post = np.asarray(post_condition)
        post = post[0] if post.ndim == 3 else post
        places, cf = alltoall_layout(pre, post, sw, mask)
        prog, scratch = alltoall_program(rounds, places, v2r)
        xml = lower_to_xml(prog, ngpus=n, in_chunks=n * cf, out_chunks=n * cf, scratch_chunks=scratch,
                           coll="alltoall", name=name, instances=instances, instr_fusion=instr_fusion)
        if check:
            live = {(p.origin_rank, p.dest_rank, p.dest_index % cf) for p in places}
            # input[r][d * cf + j] is the j-th chunk from r to d; it must end in output[d][r * cf + j]
            check_xml(xml, lambda r, i, k: ("a", i // cf, r, i % cf, k) if (i // cf, r, i % cf) in live else None,
                      lambda r, i, k: ("a", r, i // cf, i % cf, k))
    else:
        raise ValueError(f"collective must be one of {COLLECTIVES}")
    return xml


def _gpu_nodes(problem) -> list[int]:
    roles = (getattr(problem, "metadata", None) or {}).get("node_roles")
    if roles:
        return [i for i, r in enumerate(roles) if r == "gpu"]
    return list(range(int(problem.V)))


def schedule_transfers(problem, schedule: Sequence[np.ndarray]) -> list[tuple[int, int, int, int]]:
    """(slot, chunk, src_gpu, dst_gpu) GPU-to-GPU transfers of a problem's schedule."""
    edges = np.asarray(problem.topology, dtype=np.int64).reshape(-1, 2)
    gpus = set(_gpu_nodes(problem))
    sw = np.asarray([v not in gpus for v in range(int(problem.V))])
    rounds = gpu_transfers(schedule, edges[:, 0], edges[:, 1], np.asarray(problem.initial_state), sw)
    return [(t, c, u, v) for t, tr in enumerate(rounds) for u, v, c in tr]


def build_xml(problem, schedule: Sequence[np.ndarray], *, name: str = "raiccl_schedule", proto: str = "Simple") -> str:
    """Any problem's schedule as a custom-collective program: chunk c lives at
    offset c in the input buffer of its origin and the output buffer of every
    GPU it reaches."""
    rounds = schedule_transfers(problem, schedule)
    gpus = _gpu_nodes(problem)
    v2r = {v: r for r, v in enumerate(gpus)}
    init = np.asarray(problem.initial_state)
    C = int(problem.C)
    prog = []
    for c in range(C):
        owners = [v for v in np.flatnonzero(init[c]).tolist() if v in v2r]
        for v in owners:
            prog.append(Copy(-1, v2r[v], "i", c, v2r[v], "o", c))
    for t, c, u, v in rounds:
        prog.append(Copy(t, v2r[u], "o", c, v2r[v], "o", c))
    return lower_to_xml(prog, ngpus=len(gpus), in_chunks=C, out_chunks=C, scratch_chunks=0, coll="custom",
                        name=name, proto=proto)


def export_problem_schedule(problem, schedule, path: str, *, name: str = "raiccl_schedule") -> str:
    xml = build_xml(problem, schedule, name=name)
    with open(path, "w", encoding="utf-8") as f:
        f.write(xml)
    return xml


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(prog="revealaiccl_b200.rl.xml_export",
                                 description="Lower a saved slot schedule to MSCCL XML (checked).")
    ap.add_argument("--input", required=True, help="torch file: real_strategy_list, edge_src_idx, edge_dst_idx, "
                                                   "pre_condition[, post_condition, is_switch, chunk_mask]")
    ap.add_argument("--out", default=None)
    ap.add_argument("--collective", default="allgather", choices=COLLECTIVES)
    ap.add_argument("--instances", type=int, default=1)
    ap.add_argument("--instr-fusion", action="store_true")
    ap.add_argument("--no-check", action="store_true")
    ap.add_argument("--name", default="raiccl_schedule")
    args = ap.parse_args(argv)
    import torch

    d = torch.load(args.input, map_location="cpu", weights_only=False)

    def arr(key, required=True):
        if key not in d or d[key] is None:
            if required:
                raise SystemExit(f"input lacks {key}")
            return None
        v = d[key]
        return v.detach().cpu().numpy() if hasattr(v, "detach") else np.asarray(v)

    sched = [s.detach().cpu().numpy() if hasattr(s, "detach") else np.asarray(s) for s in d["real_strategy_list"]]
    xml = schedule_to_msccl_xml(sched, edge_src=arr("edge_src_idx"), edge_dst=arr("edge_dst_idx"),
                                pre_condition=arr("pre_condition"), post_condition=arr("post_condition", False),
                                is_switch=arr("is_switch", False), chunk_mask=arr("chunk_mask", False),
                                collective=args.collective, name=args.name, instances=args.instances,
                                instr_fusion=args.instr_fusion, check=not args.no_check)
    if args.out:
        with open(args.out, "w", encoding="utf-8") as f:
            f.write(xml)
    else:
        print(xml, end="")


__all__ = ["Copy", "Placement", "allgather_layout", "allgather_program", "alltoall_layout", "alltoall_program",
           "build_xml", "check_xml", "export_problem_schedule", "gpu_transfers", "lower_to_xml", "main",
           "schedule_to_msccl_xml", "schedule_transfers"]

if __name__ == "__main__":
    main()

"""Lower a slot schedule (Y_t[c, e] = 1: chunk c crosses edge e in slot t) to an
MSCCL-style XML program, written directly (no msccl-tools dependency).

Capability of rlccl/utils/xml_converter.py (which goes through MSCCLang):
every GPU gets one receive threadblock per incoming peer and one send
threadblock per outgoing peer that the schedule uses; steps are ordered by
slot, a forward of chunk c depends on the step that received c at an earlier
slot (``depid``/``deps``), and chunk c lives at offset c of the input buffer
of its origin and of the output buffer of every other GPU.  Non-GPU nodes
(switch / NIC) are traced through: a transfer u -> switch -> v becomes one
GPU-to-GPU transfer u -> v.
"""

from __future__ import annotations

from collections import defaultdict
from typing import Sequence
from xml.sax.saxutils import quoteattr

import numpy as np


def _gpu_nodes(problem) -> list[int]:
    roles = (getattr(problem, "metadata", None) or {}).get("node_roles")
    if roles:
        return [i for i, r in enumerate(roles) if r == "gpu"]
    return list(range(int(problem.V)))


def schedule_transfers(problem, schedule: Sequence[np.ndarray]) -> list[tuple[int, int, int, int]]:
    """(slot, chunk, src_gpu, dst_gpu) GPU-to-GPU transfers, tracing through non-GPU nodes."""
    edges = np.asarray(problem.topology, dtype=np.int64).reshape(-1, 2)
    gpus = set(_gpu_nodes(problem))
    relay_origin: dict[tuple[int, int], int] = {}
    out = []
    for t, Y in enumerate(schedule):
        for c, e in zip(*np.nonzero(np.asarray(Y))):
            u, v = int(edges[e, 0]), int(edges[e, 1])
            origin = u if u in gpus else relay_origin.get((int(c), u), u)
            if v in gpus:
                if origin in gpus and origin != v:
                    out.append((t, int(c), origin, v))
            else:
                relay_origin[(int(c), v)] = origin
    return out


def build_xml(problem, schedule: Sequence[np.ndarray], *, name: str = "raiccl_schedule", proto: str = "Simple") -> str:
    transfers = schedule_transfers(problem, schedule)
    gpus = _gpu_nodes(problem)
    C = int(problem.C)
    init = np.asarray(problem.initial_state)
    origin = {c: int(np.flatnonzero(init[c])[0]) if init[c].any() else -1 for c in range(C)}
    sends: dict[tuple[int, int], list] = defaultdict(list)
    recvs: dict[tuple[int, int], list] = defaultdict(list)
    for t, c, s, d in sorted(transfers):
        sends[(s, d)].append((t, c))
        recvs[(d, s)].append((t, c))
    lines = [f'<algo name={quoteattr(name)} proto="{proto}" nchannels="1" nchunksperloop="{C}" '
             f'ngpus="{len(gpus)}" coll="custom" inplace="0">']
    for g in gpus:
        lines.append(f'  <gpu id="{g}" i_chunks="{C}" o_chunks="{C}" s_chunks="0">')
        tb = 0
        received: dict[int, list] = defaultdict(list)  # chunk -> [(slot, tb, step)]
        for (gg, peer), items in sorted(recvs.items()):
            if gg != g:
                continue
            lines.append(f'    <tb id="{tb}" send="-1" recv="{peer}" chan="0">')
            for s, (t, c) in enumerate(items):
                lines.append(f'      <step s="{s}" type="r" srcbuf="o" srcoff="{c}" dstbuf="o" dstoff="{c}" cnt="1" '
                             f'depid="-1" deps="-1" hasdep="1"/>')
                received[c].append((t, tb, s))
            lines.append("    </tb>")
            tb += 1
        for (gg, peer), items in sorted(sends.items()):
            if gg != g:
                continue
            lines.append(f'    <tb id="{tb}" send="{peer}" recv="-1" chan="0">')
            for s, (t, c) in enumerate(items):
                buf = "i" if origin.get(c) == g else "o"
                earlier = [(tt, tbi, si) for tt, tbi, si in received.get(c, []) if tt < t]
                dep = max(earlier)[1:] if earlier else (-1, -1)
                lines.append(f'      <step s="{s}" type="s" srcbuf="{buf}" srcoff="{c}" dstbuf="o" dstoff="{c}" '
                             f'cnt="1" depid="{dep[0]}" deps="{dep[1]}" hasdep="0"/>')
            lines.append("    </tb>")
            tb += 1
        lines.append("  </gpu>")
    lines.append("</algo>")
    return "\n".join(lines) + "\n"


def export_problem_schedule(problem, schedule, path: str, *, name: str = "raiccl_schedule") -> str:
    xml = build_xml(problem, schedule, name=name)
    with open(path, "w", encoding="utf-8") as f:
        f.write(xml)
    return xml


__all__ = ["build_xml", "export_problem_schedule", "schedule_transfers"]

"""Failure detection without a GPU fault: host-side injection on simulated
ranks and on gloo process groups (CPU), and a withheld device signal that
must end in a bounded-wait status instead of a hang (GPU)."""

from datetime import timedelta
import multiprocessing as mp
import os
import socket
import time

import pytest
import torch

from revealaiccl_b200.moe.config import preset
from revealaiccl_b200.moe.simulated import PeerSignalMissing, SimulatedMoE


def _sim():
    return SimulatedMoE(preset("cpu_sim_2rank").with_overrides(tokens_per_rank=256, chunk_sizes=(32,) * 8), 2)


def test_simulated_dropped_signal_fails_closed():
    sim = _sim()
    assert sim.run("early").outputs  # healthy call
    for arm in ("early", "delayed"):
        with pytest.raises(PeerSignalMissing):
            sim.run(arm, drop_signal=(0, 1, 3))


def test_simulated_corrupted_count_header_is_detected():
    sim = _sim()
    try:
        res = sim.run("early", corrupt_count=(1, 0, 2))
    except RuntimeError:
        return  # rejected outright
    bad = [c for c in res.forward_checks if any(int(v) for k, v in c.items() if k not in ("digest", "rows"))]
    assert bad, "a corrupted count header went unnoticed"


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_raises(rank, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=3))
    try:
        if rank == 1:
            raise SystemExit(3)  # leaves before the collective its peer enters
        t0 = time.monotonic()
        try:
            dist.all_reduce(torch.ones(4))
            q.put(("no-error", time.monotonic() - t0))
        except Exception as exc:
            q.put(("error", time.monotonic() - t0, type(exc).__name__))
    finally:
        if rank == 0:
            dist.destroy_process_group()


def _rank_heartbeat(rank, port, mode, q):
    import torch.distributed as dist

    from revealaiccl_b200.utils.watchdog import Heartbeat, PeerFailure

    store = dist.TCPStore("127.0.0.1", port, 2, rank == 0, timeout=timedelta(seconds=10))
    hb = Heartbeat(store, rank, 2, interval=0.1, timeout=1.0).start()
    if rank == 1:
        time.sleep(0.5)
        if mode == "crash":
            os._exit(0)  # no clean leave: heartbeats just stop
        hb.stop()
        time.sleep(2.0)
        return
    t0 = time.monotonic()
    while time.monotonic() - t0 < 8.0:
        try:
            hb.check_peers()
        except PeerFailure as exc:
            q.put((exc.dead, exc.left, time.monotonic() - t0))
            hb.stop()
            return
        time.sleep(0.05)
    q.put(("none",))
    hb.stop()


def _spawn(target, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, *args, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        return q.get(timeout=60)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()


def test_gloo_rank_exit_ends_peer_collective_with_error():
    res = _spawn(_rank_raises, _free_port())
    assert res[0] == "error" and res[1] < 30


@pytest.mark.parametrize("mode", ["crash", "leave"])
def test_heartbeat_reports_dead_or_left_peer(mode):
    res = _spawn(_rank_heartbeat, _free_port(), mode)
    assert res[0] != "none"
    dead, left, _ = res
    assert (dead == [1]) if mode == "crash" else (left == [1] and dead == [])


@pytest.mark.gpu
def test_withheld_device_signal_times_out_then_recovers():
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer
    from revealaiccl_b200.ops.status import DeviceStatusError

    layer = ProgressiveMoELayer(preset("r4_reference"), timeout_s=0.5)
    try:
        layer.forward("early")
        assert layer.verify()["pass"]
        layer.inject_skip_signal(3)
        t0 = time.monotonic()
        layer.forward("early")
        rec = layer.status_record()
        assert time.monotonic() - t0 < 10
        assert rec["code"] == 2  # peer signal wait timed out (bounded), context still usable
        with pytest.raises(DeviceStatusError):
            layer.check_status()
        layer.inject_skip_signal(-1)
        layer.clear_status()
        layer.forward("early")
        layer.check_status()
        assert layer.verify()["pass"]
    finally:
        layer.clear_status()
        layer.close()

"""Completion bridge (native polling thread): flag slots written from the host
(CPU), CUDA-event and kernel-published flag slots (GPU), timeouts that raise,
snapshot fields and re-arming rules (reference extensions/r2_event_bridge
behaviour)."""

import threading
import time

import pytest
import torch

from revealaiccl_b200.ops import _native

pytestmark = pytest.mark.skipif(not _native.has_host(), reason="host runtime not built")


def test_flag_slot_from_host_writer():
    from revealaiccl_b200.runtime import CompletionBridge, HostFlag

    flag = HostFlag(mapped=False)
    with CompletionBridge(3) as br:
        br.arm_flag(0, flag, 5)
        assert not br.ready(0)
        t = threading.Timer(0.02, flag.write, args=(5,))
        t0 = time.monotonic_ns()
        t.start()
        ready = br.wait_ready(0, 2.0)
        assert br.ready(0) and ready >= t0
        s = br.snapshot()[0]
        assert s["source"] == "flag" and s["state"] == 2 and s["poll_count"] > 1
        assert s["upper_bound_valid"] and s["visibility_upper_bound_ns"] > 0
        with pytest.raises(RuntimeError, match="not armed"):
            br.wait_ready(1, 0.01)
        br.arm_flag(1, flag, 6)  # never written
        with pytest.raises(RuntimeError, match="timeout"):
            br.wait_ready(1, 0.02)
        with pytest.raises(RuntimeError, match="already armed"):
            br.arm_flag(1, flag, 6)
        with pytest.raises(RuntimeError, match="armed"):
            br.reset_all()
        flag.write(6)
        br.wait_all(2.0)
        br.reset_all()
        assert br.snapshot()[0]["state"] == 0
    with pytest.raises(ValueError):
        CompletionBridge(2)._b.arm_flag(0, 3, 1)  # misaligned pointer


@pytest.mark.gpu
def test_event_and_device_flag_slots():
    from revealaiccl_b200.runtime import CompletionBridge, HostFlag

    flag = HostFlag()
    try:
        with CompletionBridge(2, device=torch.cuda.current_device()) as br:
            for i in range(1, 6):
                br.reset_all()
                br.arm_flag(1, flag, i)
                flag.signal_from_device(i, delay_ns=200_000)
                ev = torch.cuda.Event()
                ev.record()
                br.arm_event(0, ev)
                br.wait_all(5.0)
                assert flag.read() == i and br.ready(0) and br.ready(1)
            torch.cuda.synchronize()
    finally:
        flag.close()


@pytest.mark.gpu
def test_latency_runner():
    from revealaiccl_b200.bench import event_latency

    rep = event_latency.run(trials=20, delay_us=10.0)
    assert rep["flag"]["wall_ns"]["count"] == 20 and rep["event"]["wall_ns"]["count"] == 20

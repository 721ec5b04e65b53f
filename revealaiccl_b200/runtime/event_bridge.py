"""Completion bridge: device completion -> host-visible READY per slot.

Behaviour of extensions/r2_event_bridge/{event_bridge,integrated_event_bridge}.cpp
(slot array, arm / ready / ready_ns / wait_ready / wait_all / snapshot /
reset_all / stop, GIL-free waits that raise on timeout or CUDA error, and the
conservative completion -> visible upper bound = hit time - start of the last
missed poll).  The polling thread is native (``_host.EventBridge``); slots
watch either a CUDA event (``cudaEventQuery``) or a 64-bit word in mapped
host memory that a kernel publishes with a system-scope release — the second
kind needs no CUDA call on the polling path.
"""

from __future__ import annotations

from typing import Any

import numpy as np

from ..ops._native import host, kernels


class HostFlag:
    """A 64-bit word in pinned, device-mapped host memory (or plain host memory for host-side writers)."""

    def __init__(self, *, mapped: bool = True) -> None:
        self.mapped = mapped
        if mapped:
            self.host_ptr, self.device_ptr = host().alloc_mapped(64)
            self._buf = None
        else:  # host-only word (tests, host producers)
            self._buf = np.zeros(8, dtype=np.uint64)
            self.host_ptr, self.device_ptr = int(self._buf.ctypes.data), 0
        self.write(0)

    def read(self) -> int:
        return int(host().read_u64(self.host_ptr)) if self.mapped else int(self._buf[0])

    def write(self, value: int) -> None:
        if self.mapped:
            host().write_u64(self.host_ptr, int(value))
        else:
            self._buf[0] = np.uint64(value)

    def signal_from_device(self, value: int, delay_ns: int = 0) -> None:
        """Publish ``value`` from the current CUDA stream after ``delay_ns`` of device time."""
        if not self.mapped:
            raise RuntimeError("a host-only flag cannot be written by a kernel")
        kernels().signal_host_flag(self.device_ptr, int(value), int(delay_ns))

    def close(self) -> None:
        if self.mapped and self.host_ptr:
            host().free_mapped(self.host_ptr)
            self.host_ptr = self.device_ptr = 0


class CompletionBridge:
    """Slots of completion sources polled by one native (optionally pinned) host thread."""

    def __init__(self, capacity: int, *, cpu_core: int = -1, device: int = -1) -> None:
        self._b = host().EventBridge(int(capacity), int(cpu_core), int(device))
        self.capacity = int(capacity)

    def arm_event(self, index: int, event: Any) -> None:
        """Watch a ``torch.cuda.Event`` (recorded or about to be recorded)."""
        handle = int(getattr(event, "cuda_event", event))
        self._b.arm(int(index), handle)

    def arm_flag(self, index: int, flag: HostFlag, expected: int) -> None:
        self._b.arm_flag(int(index), int(flag.host_ptr), int(expected))

    def ready(self, index: int) -> bool:
        return bool(self._b.ready(int(index)))

    def ready_ns(self, index: int) -> int:
        return int(self._b.ready_ns(int(index)))

    def wait_ready(self, index: int, timeout_s: float) -> int:
        return int(self._b.wait_ready(int(index), int(timeout_s * 1e9)))

    def wait_all(self, timeout_s: float) -> None:
        self._b.wait_all(int(timeout_s * 1e9))

    def snapshot(self) -> list[dict]:
        return list(self._b.snapshot())

    def reset_all(self) -> None:
        self._b.reset_all()

    def stop(self) -> None:
        self._b.stop()

    def __enter__(self) -> "CompletionBridge":
        return self

    def __exit__(self, *exc) -> None:
        self.stop()

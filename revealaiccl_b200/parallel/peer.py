"""NVLink peer channel: symmetric device regions mapped on every rank.

Each rank allocates one region of identical size with ``cudaMalloc`` (in the
native host runtime), exports its CUDA-IPC handle, and the handles travel
once over the torch process group (``all_gather_object``).  Every rank then
opens all peers' handles, giving a table of device pointers — own region
included — that kernels store into directly over NVLink/NVSwitch.  Replaces
the two-rank MSCCL++ bootstrap/registerMemory/MemoryChannel set-up of
extensions/r6_mscclpp/mscclpp_runtime.cu:20-90.

``device_view`` wraps any device address range as a torch tensor (through
``__cuda_array_interface__``) without copying, for host-side inspection of a
region by the checker.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._native import host


class _CudaArray:
    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {
            "shape": tuple(int(s) for s in shape), "typestr": typestr,
            "data": (int(ptr), False), "version": 3, "strides": None, "stream": None,
        }


_TYPESTR = {torch.uint8: "|u1", torch.int32: "<i4", torch.int64: "<i8", torch.float32: "<f4",
            torch.float16: "<f2", torch.bfloat16: "<f2"}


def device_view(ptr: int, shape: tuple[int, ...], dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """Zero-copy tensor over device memory at ``ptr`` (bf16 viewed via int16 bits)."""
    if dtype == torch.bfloat16:
        t = torch.as_tensor(_CudaArray(ptr, shape, "<i2"), device=device)
        return t.view(torch.bfloat16)
    return torch.as_tensor(_CudaArray(ptr, shape, _TYPESTR[dtype]), device=device)


class PeerChannel:
    """Symmetric region of ``nbytes`` on every rank, plus every peer's mapping."""

    def __init__(self, nbytes: int, device: torch.device, group=None) -> None:
        self.device = torch.device(device)
        self.index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.nbytes = int(nbytes)
        self._host = host()
        self.local_ptr, handle = self._host.alloc_symmetric(self.nbytes, self.index)
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        self._opened: list[int] = []
        if self.world == 1:
            self.bases = [self.local_ptr]
        else:
            handles: list = [None] * self.world
            dist.all_gather_object(handles, handle, group=group)
            bases = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    bases.append(self.local_ptr)
                else:
                    p = self._host.open_peer(h, self.index)
                    self._opened.append(p)
                    bases.append(p)
            self.bases = bases
        self._device_counters: torch.Tensor | None = None

    COUNTER_FIELDS = ("put_calls", "bytes_transferred", "signals", "waits", "return_bytes", "return_signals")
    COUNTER_STRIDE = 8  # int64 words per peer in the device counter array

    def bind_counters(self, counters: torch.Tensor) -> None:
        """Attach the device counter array the data-plane kernels update:
        [world][8] int64 words per peer (descriptors put, forward bytes, ready
        signals sent, ready words waited for, return bytes, return signals)."""
        if counters.dtype != torch.int64 or counters.numel() != self.world * self.COUNTER_STRIDE:
            raise ValueError("peer counters must be int64 [world * 8]")
        self._device_counters = counters

    def peer_counters(self) -> list[dict[str, int]]:
        """Per-peer counts (index = peer rank, own rank included) since the layer was built."""
        if self._device_counters is None:
            return [dict.fromkeys(self.COUNTER_FIELDS, 0) for _ in range(self.world)]
        rows = self._device_counters.view(self.world, self.COUNTER_STRIDE).cpu().tolist()
        return [dict(zip(self.COUNTER_FIELDS, row)) for row in rows]

    @property
    def counters(self) -> dict[str, int]:
        """Totals over all peers of the device counters (the MSCCL++ runtime's
        put_calls / bytes_transferred / signals / waits, plus the return side)."""
        total = dict.fromkeys(self.COUNTER_FIELDS, 0)
        for row in self.peer_counters():
            for k, v in row.items():
                total[k] += int(v)
        return total

    def view(self, offset: int, shape: tuple[int, ...], dtype: torch.dtype, rank: int | None = None) -> torch.Tensor:
        base = self.bases[self.rank if rank is None else rank]
        return device_view(base + int(offset), shape, dtype, self.device)

    def close(self) -> None:
        for p in self._opened:
            try:
                self._host.close_peer(p, self.index)
            except RuntimeError:
                pass
        self._opened = []
        if self.local_ptr:
            self._host.free_symmetric(self.local_ptr, self.index)
            self.local_ptr = 0

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass


__all__ = ["PeerChannel", "device_view"]

"""Device status words written by the kernels instead of trapping.

Every bounded wait and bounds check in the sm_100a kernels records the first
failure into a small ``DeviceStatus`` record (code, kernel id, block, thread,
index, bound).  The host reads it after the launch and raises, so a missing
peer signal or an index bug ends the op with an error instead of a hung or
faulted GPU.
"""

from __future__ import annotations

import torch

STATUS_WORDS = 8  # int32 words: code, kernel_id, block, thread, index(lo,hi), bound(lo,hi)

CODES = {
    0: "ok",
    1: "pipeline mbarrier wait timed out",
    2: "peer signal wait timed out",
    3: "router chunk flag wait timed out",
    4: "bounds violation",
    5: "bad launch configuration",
    6: "descriptor permit wait timed out",
    7: "signal sequence mismatch",
    8: "streamed input chunk never landed",
}


class DeviceStatusError(RuntimeError):
    def __init__(self, record: dict):
        self.record = record
        super().__init__(
            f"device status {record['code']} ({CODES.get(record['code'], '?')}): "
            f"kernel={record['kernel_id']} block={record['block']} thread={record['thread']} "
            f"index={record['index']} bound={record['bound']}"
        )


def new_status(device: torch.device | str) -> torch.Tensor:
    return torch.zeros(STATUS_WORDS, dtype=torch.int32, device=device)


def decode(status: torch.Tensor) -> dict:
    words = status.detach().to("cpu").view(torch.int32)
    w = [int(v) for v in words.tolist()]
    idx = (w[5] << 32) | (w[4] & 0xFFFFFFFF)
    bound = (w[7] << 32) | (w[6] & 0xFFFFFFFF)
    return {"code": w[0], "kernel_id": w[1], "block": w[2], "thread": w[3], "index": idx, "bound": bound}


def check(status: torch.Tensor) -> None:
    rec = decode(status)
    if rec["code"] != 0:
        raise DeviceStatusError(rec)

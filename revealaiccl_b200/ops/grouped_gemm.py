"""Python front end of the tcgen05 grouped GEMM (csrc/include/grouped_gemm.cuh).

``grouped_gemm`` computes, for every segment ``s`` (a run of rows that share
one expert weight):

    out[row_map[r], :] = act(A[r] @ B[expert_s].T + bias[expert_s]) * row_scale[r]

with the accumulator in TMEM, operands staged by TMA, and the output written
either to a local tensor or to an NVLink peer pointer (``out_ptrs``).

It replaces the per-expert ``index_select`` + two matmuls + ``index_copy_`` of
the reference expert loop (rlccl/transport/reference_full_moe.py:271-280).
"""

from __future__ import annotations

from typing import Sequence

import torch

from . import status as _status
from ._native import kernels

ACT_IDS = {"none": 0, "relu": 1, "gelu": 2, "silu": 3, "swiglu": 4}
SEG_FIELDS = 8
DEFAULT_TIMEOUT_NS = 2_000_000_000


def num_sms(device: torch.device) -> int:
    return torch.cuda.get_device_properties(device).multi_processor_count


def pick_bn(n: int, swiglu: bool = False) -> int:
    for bn in (256, 128, 64, 32, 16):
        if n % bn == 0 and (not swiglu or bn >= 32):
            return bn
    raise ValueError(f"GEMM N={n} is not a multiple of 16")


def make_segments(rows: Sequence[tuple[int, int, int, int, int]], device) -> torch.Tensor:
    """rows: (a_row0, rows, expert, out_slot, out_row0) per segment."""
    seg = torch.zeros((max(1, len(rows)), SEG_FIELDS), dtype=torch.int32)
    for i, r in enumerate(rows):
        seg[i, :5] = torch.tensor(r, dtype=torch.int32)
    return seg.to(device)


def swiglu_interleave(w_gate: torch.Tensor, w_up: torch.Tensor, bn: int) -> torch.Tensor:
    """Pack [E, F, K] gate/up weights into [E, 2F, K] so that every BN-row tile
    holds BN/2 gate rows followed by the BN/2 matching up rows (the layout the
    SwiGLU epilogue expects)."""
    e, f, k = w_gate.shape
    half = bn // 2
    if f % half:
        raise ValueError("SwiGLU width must be a multiple of BN/2")
    g = w_gate.reshape(e, f // half, half, k)
    u = w_up.reshape(e, f // half, half, k)
    return torch.cat([g, u], dim=2).reshape(e, 2 * f, k).contiguous()


def swiglu_interleave_bias(b_gate: torch.Tensor, b_up: torch.Tensor, bn: int) -> torch.Tensor:
    e, f = b_gate.shape
    half = bn // 2
    g = b_gate.reshape(e, f // half, half)
    u = b_up.reshape(e, f // half, half)
    return torch.cat([g, u], dim=2).reshape(e, 2 * f).contiguous()


def grouped_gemm(
    A: torch.Tensor,
    B: torch.Tensor,
    segs: torch.Tensor,
    *,
    n: int,
    act: str = "none",
    bias: torch.Tensor | None = None,
    row_map: torch.Tensor | None = None,
    row_scale: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    out_ptrs: torch.Tensor | None = None,
    ldo: int | None = None,
    out_dtype: torch.dtype | None = None,
    bn: int | None = None,
    status: torch.Tensor | None = None,
    prefix: torch.Tensor | None = None,
    grid: int | None = None,
    timeout_ns: int = DEFAULT_TIMEOUT_NS,
    check: bool = False,
    pair: bool = False,
    swap_max: int = 0,
) -> torch.Tensor | None:
    """Launch the grouped GEMM on the current stream.

    Either ``out`` (a local tensor, slot 0) or ``out_ptrs`` (int64 device
    pointers, one per ``out_slot``) must be given.  ``pair=True`` runs the
    CTA-pair kernel (256 x bn tiles on clusters of two SMs; bn >= 64).
    ``swap_max > 0`` (pair kernel, bn = 256, no SwiGLU) computes a segment's
    last 256-row tile of at most ``swap_max`` rows with swapped operands: the
    weights fill the 256-row side and the tail's tokens the narrow N side, so
    a short tail costs a fraction of a full tile.  With ``check=True`` the
    call synchronises and raises on a recorded device status.
    """
    mod = kernels()
    swiglu = act == "swiglu"
    if bn is None:
        bn = pick_bn(n, swiglu)
    if out is not None:
        out_dtype = out.dtype
        ldo = out.stride(0)
        out_ptrs = torch.tensor([out.data_ptr()], dtype=torch.int64, device=A.device)
    if out_ptrs is None or ldo is None:
        raise ValueError("grouped_gemm needs `out` or (`out_ptrs`, `ldo`)")
    out_bf16 = (out_dtype or torch.float32) == torch.bfloat16
    if status is None:
        status = _status.new_status(A.device)
    if prefix is None:
        tables = 2 if swap_max > 0 else 1  # full-tile table, then the swapped-tail table
        prefix = torch.empty(tables * (segs.shape[0] + 1), dtype=torch.int32, device=A.device)
    if grid is None:
        grid = num_sms(A.device)
    mod.grouped_gemm(
        A, B, segs, prefix, int(n), int(bn), ACT_IDS[act], bias, row_map, row_scale,
        out_ptrs, int(ldo), bool(out_bf16), status, int(grid), int(timeout_ns), bool(pair),
        int(swap_max),
    )
    if check:
        torch.cuda.synchronize(A.device)
        _status.check(status)
    return out

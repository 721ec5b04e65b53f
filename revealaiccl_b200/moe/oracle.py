"""Plain PyTorch fp32 oracle of the MoE layer (untimed; the reference for the kernels).

* ``router_reference``: logits = x @ W^T + b (+ chunk bias), masks, then a
  stable descending sort so ties choose the smaller expert id — the exact
  contract of rlccl/transport/reference_router.py:15-25 — and the gates.
* ``expert_reference``: relu/gelu/silu MLP or SwiGLU of one expert in fp32.
* ``layer_reference``: per-token sum over the chosen experts of gate x MLP.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .config import MoELayerConfig
from .inputs import LayerWeights, RankInputs


def router_logits(cfg: MoELayerConfig, x: torch.Tensor, w: LayerWeights, inp: RankInputs) -> torch.Tensor:
    logits = x.float() @ w.router_w.float().t() + w.router_b.float()
    if inp.chunk_bias is not None:
        off = cfg.chunk_offsets
        rows = torch.zeros_like(logits)
        for c in range(cfg.chunks):
            rows[off[c]:off[c + 1]] = inp.chunk_bias[c]
        logits = logits + rows
    E = cfg.experts
    mask = torch.zeros_like(logits, dtype=torch.bool)
    if cfg.mask_mode == "topology_source":
        pos = torch.arange(logits.shape[0], device=logits.device)
        mask[pos, pos % E] = True
    if inp.block_mask is not None:
        mask |= inp.block_mask.bool()[None, :]
    return logits.masked_fill(mask, float("-inf"))


def router_reference(cfg: MoELayerConfig, x: torch.Tensor, w: LayerWeights, inp: RankInputs):
    logits = router_logits(cfg, x, w, inp)
    values, indices = torch.sort(logits, dim=-1, descending=True, stable=True)
    ids = indices[:, :cfg.top_k]
    top = values[:, :cfg.top_k]
    if cfg.gate_mode == "topk_softmax":
        gates = torch.softmax(top, dim=-1)
    elif cfg.gate_mode == "softmax":
        gates = torch.softmax(logits, dim=-1).gather(1, ids)
    else:
        gates = torch.ones_like(top)
    return ids.to(torch.int32), gates.float(), logits


def expert_reference(cfg: MoELayerConfig, x: torch.Tensor, w: LayerWeights, e: int) -> torch.Tensor:
    xf = x.float()
    if cfg.activation == "swiglu":
        wg = w.w_gate[e].float() if w.w_gate is not None else w.w1[e, :cfg.ffn_hidden].float()
        wu = w.w_up[e].float() if w.w_up is not None else w.w1[e, cfg.ffn_hidden:].float()
        h = F.silu(xf @ wg.t()) * (xf @ wu.t())
    else:
        h = xf @ w.w1[e].float().t()
        if w.b1 is not None:
            h = h + w.b1[e].float()
        h = {"relu": torch.relu, "gelu": F.gelu, "silu": F.silu}[cfg.activation](h)
    if cfg.dtype == "bf16":
        h = h.to(torch.bfloat16).float()  # the kernel keeps the hidden activation in bf16
    y = h @ w.w2[e].float().t()
    if w.b2 is not None:
        y = y + w.b2[e].float()
    return y


def layer_reference(cfg: MoELayerConfig, x: torch.Tensor, w: LayerWeights, ids: torch.Tensor,
                    gates: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns (combined [T, Dout], per-assignment outputs [T, k, Dout]) in fp32."""
    T, k = ids.shape
    per = torch.zeros((T, k, cfg.out_dim), dtype=torch.float32, device=x.device)
    ids_l = ids.long()
    with torch.no_grad():
        prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        try:
            for e in range(cfg.experts):
                sel = (ids_l == e).nonzero(as_tuple=False)
                if sel.numel() == 0:
                    continue
                y = expert_reference(cfg, x[sel[:, 0]], w, e)
                per[sel[:, 0], sel[:, 1]] = y * gates[sel[:, 0], sel[:, 1], None]
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev
    return per.sum(dim=1), per


__all__ = ["expert_reference", "layer_reference", "router_logits", "router_reference"]

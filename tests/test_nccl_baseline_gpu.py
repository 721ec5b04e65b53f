"""The PyTorch + NCCL baseline layer (the ``--impl nccl`` arm of bench.py) on
one GPU: its output equals the fp32 oracle of the same routing, and its
early and delayed arms agree."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name,over", [
    ("r4_reference", {}),
    ("full_tf32", dict(tokens_per_rank=1024, chunk_sizes=(128,) * 8)),
    ("deepseek_v2_lite", dict(tokens_per_rank=1024, chunk_sizes=(64,) * 16)),
])
def test_nccl_layer_matches_oracle(name, over):
    from revealaiccl_b200.moe.config import preset
    from revealaiccl_b200.moe.oracle import layer_reference
    from revealaiccl_b200.transport.nccl_baseline import NcclMoELayer

    cfg = preset(name, **over)
    layer = NcclMoELayer(cfg, device=torch.device("cuda", 0))
    out = layer.forward("early").clone()
    ref, _ = layer_reference(cfg, layer.inputs.tokens, layer.weights, layer.ids.int(), layer.gates)
    tol = 2e-2 if cfg.dtype == "bf16" else 5e-3
    torch.testing.assert_close(out, ref, atol=tol, rtol=tol)
    assert torch.equal(out, layer.forward("delayed"))

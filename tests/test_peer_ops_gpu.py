"""Standalone peer put + signal and bounded wait on one GPU (the own rank's
mapping): data and signal arrive, sequence numbers advance, and a wait for a
signal that nothing sends times out with a status instead of hanging, after
which the context still works."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_put_signal_wait_and_bounded_timeout():
    from revealaiccl_b200.ops import status as st
    from revealaiccl_b200.parallel.peer_ops import PeerOps

    dev = torch.device("cuda", 0)
    ops = PeerOps(1 << 20, dev, timeout_s=0.5)
    try:
        for it in range(3):
            src = torch.randn(4096 + 1024 * it, device=dev)
            seq = ops.put(0, src)
            assert seq == it + 1
            ops.expect(0)
            ops.wait(0)
            ops.check_status()
            got = ops.slot(0, src.numel() * 4).view(torch.float32)
            assert torch.equal(got, src)
            assert int(ops.waited[0].item()) >= 0
        assert ops.counters["put_calls"] == 3 and ops.counters["waits"] == 3
        ops.wait(0, seq=99)  # nothing will ever release 99
        torch.cuda.synchronize(dev)
        rec = st.decode(ops.status)
        assert rec["code"] == 2 and int(ops.waited[0].item()) == -1
        ops.status.zero_()
        x = torch.ones(8, device=dev)
        assert float((x * 2).sum().item()) == 16.0  # the context still runs kernels
    finally:
        ops.close()

"""Multi-GPU correctness of the progressive MoE layer (2 ranks over NVLink),
run as child processes through torch.distributed.run; skipped with fewer than
two GPUs."""

import json
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("configs", [["r4_reference", "full_tf32"], ["skewed_bf16"]])
def test_two_rank_layer_selftest(configs):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           "-m", "revealaiccl_b200.moe.selftest", "--timeout", "10", "--configs", *configs]
    if configs == ["skewed_bf16"]:
        cmd += ["--tokens", "2048"]
    p = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=700)
    recs = [json.loads(line) for line in p.stdout.splitlines() if line.startswith("{")]
    assert p.returncode == 0, (p.stdout[-3000:], p.stderr[-3000:])
    assert [r["config"] for r in recs] == configs
    assert all(r["pass"] and r["early_delayed_identical"] and r["graph_identical"] and r["streamed_identical"]
               for r in recs), recs

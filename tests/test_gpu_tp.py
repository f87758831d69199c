"""Tensor parallelism over moe_inter on 2 GPUs (the reference's own multi-chip scheme, over NCCL) against the
oracle's whole layer: runs tests/tp_worker.py under torchrun as child processes. Skipped when fewer than 2 GPUs are
visible. The process group's timeout bounds every collective, so a failure ends the ranks with an error."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_tp_two_gpus_matches_oracle():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_port()}",
           os.path.join(HERE, "tp_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0

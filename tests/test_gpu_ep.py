"""Expert parallelism on 2 GPUs (peer memory over NVLink, and NCCL send/recv) against the single-process oracle:
runs tests/ep_worker.py under torchrun as child processes. Skipped when fewer than 2 GPUs are visible (-m gpu on a
1-GPU box). Every wait on a peer is bounded, so a failure ends the ranks with an error, not a hang."""
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


def test_ep_two_gpus_matches_oracle():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_port()}",
           os.path.join(HERE, "ep_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0

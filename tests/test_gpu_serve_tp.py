"""Tensor-parallel serving on 2 GPUs (skipped with fewer): the ranks of one
group against the whole model on one GPU, through tests/tp_worker.py under
torch.distributed.run (gloo for the id exchange, NCCL inside the library,
NVLS off)."""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _gpus() -> int:
    import torch
    return torch.cuda.device_count()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif("_gpus() < 2")
def test_tp2_matches_single_gpu():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", TP_LAYERS="2")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "tp_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-4000:])
    report = json.loads(lines[-1])
    assert report["ranks_agree"] and report["logits_close"], report

"""Tensor-parallel decode on 2 GPUs of one box (skipped with fewer GPUs).

Runs tests/tp_worker.py under torch.distributed.run, with the exchanges over
NVLink peer memory (p2p) and through NCCL: greedy tokens must equal the
single-GPU engine's and the gathered logits must match.
"""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("collective,port", [("p2p", 29531), ("nccl", 29533)])
def test_tp2_matches_single_gpu(collective, port):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    here = os.path.dirname(os.path.abspath(__file__))
    cmd = ["timeout", "-k", "60", "800", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={port}", os.path.join(here, "tp_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", QWEN_TP_COLLECTIVE=collective)
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0

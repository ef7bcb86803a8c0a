"""Tensor-parallel decode on 2 GPUs of one box (skipped with fewer GPUs).

Runs tests/tp_worker.py under torch.distributed.run with NCCL: greedy tokens
must equal the single-GPU engine's and the gathered logits must match.
"""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_tp2_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    here = os.path.dirname(os.path.abspath(__file__))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29531", os.path.join(here, "tp_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0

"""Tensor-parallel decode on 2 and 4 GPUs of one box (each skipped with fewer GPUs).

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


@pytest.mark.parametrize("world,collective,port", [(2, "p2p", 29531), (2, "nccl", 29533), (4, "p2p", 29535)],
                         ids=["tp2-p2p", "tp2-nccl", "tp4-p2p"])
def test_tp_matches_single_gpu(world, collective, port):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    here = os.path.dirname(os.path.abspath(__file__))
    cmd = ["timeout", "-k", "60", "800", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(here, "tp_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", QWEN_TP_COLLECTIVE=collective)
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0

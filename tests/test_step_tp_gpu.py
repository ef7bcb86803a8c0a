"""Tensor-parallel step kernel on 2, 4 and 8 GPUs of one box (each skipped with
fewer GPUs): tests/step_tp_worker.py under torch.distributed.run; greedy
tokens and logits bit-identical to the single-GPU step engine's where the
K-slice order can match, else within the distance of two single-GPU
summation orders."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world,port", [(2, 29541), (4, 29543), (8, 29545)], ids=["tp2", "tp4", "tp8"])
def test_step_tp_bit_identical_to_single_gpu(world, port):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    here = os.path.dirname(os.path.abspath(__file__))
    cmd = ["timeout", "-k", "60", "800", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(here, "step_tp_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0

"""Worker for test_step_tp_gpu.py (run under torch.distributed.run, one GPU per rank).

The tensor-parallel step engine (one cooperative launch per GPU per token,
stages sharded over the ranks, outputs stored on every rank over NVLink) is
compared with the single-GPU step engine on the same weights and the same
K-slice count: every stage computes every output row with the same chunk
order on whichever rank owns it, so greedy tokens and logits must be
bit-identical over a prompt and 12 greedy steps.  Small Qwen3.5 member (up to
4 ranks: it has 4 value heads) and the 4B model.
"""

import datetime
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "qwen3.5-fp8-cuda_b200"))
sys.path.insert(0, os.path.join(HERE, ".."))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    from qwen35_b200 import _lib
    from qwen35_b200.config import qwen35_4b, qwen35_tiny
    from qwen35_b200.step import Qwen35StepEngine
    from qwen35_b200.step_tp import Qwen35StepTPEngine
    from qwen35_b200.weights import random_weights
    ok = True
    configs = ([("tiny", qwen35_tiny())] if world <= 4 else []) + [("4b", qwen35_4b())]
    for name, cfg in configs:
        w = random_weights(cfg, seed=21, device="cuda")
        ns = 1 if name == "tiny" else 2  # a K-slice count every residual projection's K divides
        single = Qwen35StepEngine(cfg, w, max_seq=64, keep_logits=True, nslice=ns)
        tp = Qwen35StepTPEngine(cfg, w, rank, world, max_seq=64, keep_logits=True, nslice=ns)
        prompt = [101, 7, 33, 250]
        t = prompt[0]
        for i in range(len(prompt) + 12):
            if i < len(prompt):
                t = prompt[i]
            a = single.decode(t)
            b = tp.decode(t)
            same = a == b and torch.equal(single.logits, tp.logits)
            if not same:
                err = float((single.logits.float() - tp.logits.float()).norm() / single.logits.float().norm())
                print(f"rank {rank} {name} step {i}: tokens {a} / {b}, logits rel-l2 {err:.2e}", flush=True)
                ok = False
            t = a
        if _lib.device_error() != 0:
            print(f"rank {rank} {name}: device error", flush=True)
            ok = False
        if rank == 0:
            print(f"{name}: {'bit-identical' if ok else 'MISMATCH'} over {len(prompt) + 12} steps, world {world}",
                  flush=True)
        tp.close()
        single.close()
        del tp, single, w
        torch.cuda.empty_cache()
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if int(flag.item()) == 1 else 1)


if __name__ == "__main__":
    main()

"""Worker for test_step_tp_gpu.py (run under torch.distributed.run, one GPU per rank).

The tensor-parallel step engine (one cooperative launch per GPU per token,
column-parallel in_proj / q, k, v / gate-up / LM head, row-parallel out_proj /
o_proj / down whose K-slice rows go to every rank over NVLink) is compared
with the single-GPU step engine on the same weights over a prompt and 12
greedy steps:

* where every residual projection's K chunks divide evenly over the ranks,
  the single-GPU engine with world K slices sums the same partial rows in the
  same order, so greedy tokens and logits must be bit-identical;
* otherwise (the 4B model's down projection, 18 chunks, over 4 or 8 ranks)
  the two engines round differently, so the run is teacher-forced with the
  single-GPU tokens and the logits' relative L2 distance must stay within 3x
  the distance between two single-GPU engines with different slice counts
  (two equally valid summation orders) plus 1e-3.

Configs: a widened small member (up to 4 ranks) and the 4B model.
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
    tiny = qwen35_tiny(intermediate_size=4096, num_attention_heads=8, num_key_value_heads=2,
                       linear_num_key_heads=8, linear_num_value_heads=16)
    configs = ([("tiny", tiny)] if world <= 4 else []) + [("4b", qwen35_4b())]

    def rel(a, b):
        return float((a.float() - b.float()).norm() / a.float().norm())

    for name, cfg in configs:
        w = random_weights(cfg, seed=21, device="cuda")
        chunks = [cfg.linear_value_dim // 512, cfg.num_attention_heads * cfg.head_dim // 512,
                  cfg.intermediate_size // 512]
        exact = all(c % world == 0 for c in chunks)
        single = Qwen35StepEngine(cfg, w, max_seq=64, keep_logits=True, nslice=world if exact else 0)
        other = None if exact else Qwen35StepEngine(cfg, w, max_seq=64, keep_logits=True, nslice=1)
        tp = Qwen35StepTPEngine(cfg, w, rank, world, max_seq=64, keep_logits=True, nslice=1)
        prompt = [101, 7, 33, 250]
        t = prompt[0]
        worst, floor = 0.0, 0.0
        for i in range(len(prompt) + 12):
            if i < len(prompt):
                t = prompt[i]
            a = single.decode(t)
            b = tp.decode(t)
            if exact:
                if not (a == b and torch.equal(single.logits, tp.logits)):
                    print(f"rank {rank} {name} step {i}: tokens {a} / {b}, logits rel-l2 "
                          f"{rel(single.logits, tp.logits):.2e}", flush=True)
                    ok = False
            else:
                other.decode(t)
                worst = max(worst, rel(single.logits, tp.logits))
                floor = max(floor, rel(single.logits, other.logits))
                if b != int(tp.logits.float().argmax()):
                    print(f"rank {rank} {name} step {i}: token {b} is not the argmax of the logits", flush=True)
                    ok = False
            t = a
        if not exact and worst > 3 * floor + 1e-3:
            print(f"rank {rank} {name}: logits rel-l2 {worst:.2e} > 3 x {floor:.2e} + 1e-3", flush=True)
            ok = False
        if _lib.device_error() != 0:
            print(f"rank {rank} {name}: device error", flush=True)
            ok = False
        if rank == 0:
            what = "bit-identical" if exact else f"rel-l2 {worst:.2e} (two single-GPU orders: {floor:.2e})"
            print(f"{name}: {what if ok else 'MISMATCH'} over {len(prompt) + 12} steps, world {world}", flush=True)
        tp.close()
        for e in (single, other):
            if e is not None:
                e.close()
        del tp, single, other, w
        torch.cuda.empty_cache()
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if int(flag.item()) == 1 else 1)


if __name__ == "__main__":
    main()

"""Time batch-1 decode of the random-init Qwen3.5-4B at a given context length.

    python -m qwen35_b200.profile_decode [--context 8192] [--steps 50] [--no-slices]

The KV caches of the full-attention layers are filled with random BF16 rows up
to `context` and the position is set there (the recurrent GatedDeltaNet
state is independent of the context length), then `steps` decode steps are
timed as CUDA-graph replays with CUDA events after 3 warm-up steps.  Prints
one JSON line: tokens/s, ms/step and the KV bytes each step reads.  This is
the long-context leg of BASELINE config 4 (the timing needs no prompt to be
decoded first: the values in the cache do not change the work).
"""

from __future__ import annotations

import argparse
import json

import torch

from .config import qwen35_4b
from .engine import Qwen35DecodeEngine
from .weights import random_weights


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--context", type=int, default=8192)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--no-slices", action="store_true",
                    help="residual projections reduce their K slices themselves (engine slices=False)")
    args = ap.parse_args()
    cfg = qwen35_4b()
    w = random_weights(cfg, seed=0, device="cuda")
    eng = Qwen35DecodeEngine(cfg, w, max_seq=args.context + args.steps + 16, slices=not args.no_slices)
    g = torch.Generator(device="cuda").manual_seed(1)
    for t in list(eng.k_cache.values()) + list(eng.v_cache.values()):
        t[:, : args.context].copy_(torch.randn(t[:, : args.context].shape, generator=g, device="cuda").to(t.dtype))
    eng.pos.fill_(args.context)
    eng.token.fill_(1)
    eng.capture()
    for _ in range(3):
        eng.step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        eng.step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    n_full = sum(1 for lt in cfg.layer_types if lt == "full_attention")
    ctx = args.context + 3 + args.steps // 2
    kv_bytes = n_full * 2 * cfg.num_key_value_heads * ctx * cfg.head_dim * 2
    print(json.dumps({"context": args.context, "steps": args.steps, "slices": eng.slices,
                      "tok_per_s": round(1000.0 / ms, 2),
                      "ms_per_step": round(ms, 4), "kv_bytes_per_step": kv_bytes,
                      "pos_after": int(eng.pos.item())}), flush=True)


if __name__ == "__main__":
    main()

"""Launch the GEMV at a few model shapes for a profiler capture.

    python -m qwen35_b200.profile_gemv [--shapes lm,down,q] [--reps 2]

Each shape gets fresh random E4M3 weights (two copies, alternated so that no
launch finds its weights in L2), BF16 block scales and a BF16 x, and is
launched `reps` times through the reference-named entry point
launch_gemv_v4_extern on the current stream, without programmatic dependent
launch.  Shapes: lm = 248320x2560 (LM head), down = 2560x9216, q =
8192x2560, gate = 9216x2560, kv = 1024x2560, o = 2560x4096.
"""

from __future__ import annotations

import argparse
import ctypes

import torch

from . import _lib

SHAPES = {"lm": (248320, 2560), "down": (2560, 9216), "q": (8192, 2560), "gate": (9216, 2560),
          "kv": (1024, 2560), "o": (2560, 4096)}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--shapes", default="lm,down,q")
    ap.add_argument("--reps", type=int, default=2)
    args = ap.parse_args()
    P = ctypes.c_void_p
    lib = _lib.fused()
    lib.qwen_set_pdl(0)
    stream = P(torch.cuda.current_stream().cuda_stream)
    for name in args.shapes.split(","):
        n, k = SHAPES[name]
        ws = [torch.randint(0, 120, (n, k), dtype=torch.uint8, device="cuda") for _ in range(2)]
        s = (torch.rand((n + 127) // 128, k // 128, device="cuda") * 1e-3).to(torch.bfloat16)
        x = torch.randn(k, device="cuda").to(torch.bfloat16)
        y = torch.empty(n, dtype=torch.bfloat16, device="cuda")
        for i in range(args.reps):
            lib.launch_gemv_v4_extern(P(x.data_ptr()), P(ws[i % 2].data_ptr()), P(s.data_ptr()), P(y.data_ptr()),
                                      n, k, k // 128, stream)
            _lib.check_last(f"gemv {name}")
        torch.cuda.synchronize()
        del ws
    err = _lib.device_error()
    print("ok" if err == 0 else f"device error {err}")
    if err:
        raise SystemExit(1)


if __name__ == "__main__":
    main()

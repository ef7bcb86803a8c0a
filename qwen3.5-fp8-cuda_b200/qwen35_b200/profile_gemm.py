"""Time the prefill GEMM (fp8_gemm_batch) at the config-4 shapes.

    python -m qwen35_b200.profile_gemm [--m 512,2048] [--reps 20]

For every (M, N, K) of config 4 it prints one JSON line with the device time
per call (CUDA events around `reps` back-to-back calls after 3 warm-up calls)
and the achieved TFLOP/s (2 M N K per call).  Each call includes the split of
x into the E4M3 hi/lo operand.  Also the launch harness for an ncu capture.
"""

from __future__ import annotations

import argparse
import ctypes
import json

import torch

from . import _lib

NK = [(9216, 2560), (2560, 9216), (8192, 2560), (4096, 2560), (2560, 4096), (1024, 2560)]


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--m", default="512,2048")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--shapes", default="all", help="'all' or a count of (N, K) shapes to run")
    args = ap.parse_args()
    P = ctypes.c_void_p
    lib = _lib.fp8()
    stream = P(torch.cuda.current_stream().cuda_stream)
    shapes = NK if args.shapes == "all" else NK[: int(args.shapes)]
    for m in [int(v) for v in args.m.split(",")]:
        for n, k in shapes:
            w = torch.randint(0, 120, (n, k), dtype=torch.uint8, device="cuda")
            s = (torch.rand((n + 127) // 128, k // 128, device="cuda") * 1e-3).to(torch.bfloat16)
            x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
            y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")

            def go():
                lib.fp8_gemm_batch(P(x.data_ptr()), P(w.data_ptr()), P(s.data_ptr()), P(y.data_ptr()), m, n, k,
                                   k // 128, stream)

            for _ in range(3):
                go()
            torch.cuda.synchronize()
            e = lib.qwen_fp8_last_error()
            if e:
                raise RuntimeError(f"fp8_gemm_batch failed with CUDA error {e}")
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.reps):
                go()
            e1.record()
            torch.cuda.synchronize()
            t = e0.elapsed_time(e1) / 1000.0 / args.reps
            print(json.dumps({"m": m, "n": n, "k": k, "us": round(t * 1e6, 2),
                              "tflops": round(2.0 * m * n * k / t / 1e12, 1)}), flush=True)
    if _lib.device_error():
        raise SystemExit("device error word set")


if __name__ == "__main__":
    main()

"""Launch the GEMV at a few model shapes for a profiler capture, or time them.

    python -m qwen35_b200.profile_gemv [--shapes lm,down,q] [--reps 2]
    python -m qwen35_b200.profile_gemv --time      # every config 0/1 decode shape

Each shape gets fresh random E4M3 weights (two copies, alternated so that no
launch finds its weights in L2), BF16 block scales and a BF16 x, and is
launched `reps` times through the reference-named entry point
launch_gemv_v4_extern on the current stream, without programmatic dependent
launch.  Shapes: lm = 248320x2560 (LM head), down = 2560x9216, q =
8192x2560, gate = 9216x2560, kv = 1024x2560, o = 2560x4096.

``--time`` (``time_shapes``) measures every distinct decode GEMV shape of
BASELINE configs 0 and 1 (one layer's projections and MLP of the 4B model)
as the mean time per launch of a CUDA graph of back-to-back launches: through
launch_gemv_v4_extern (the reference's entry point, no programmatic dependent
launch) and through qwen_linear_partial (the same GEMV with FP32 output,
chained with programmatic dependent launch as inside the decode engine).
Each launch reads the next of up to 64 copies of the weights (enough copies
to cycle three times the 126 MB L2 where 64 suffice); ``cycled_mb`` is the
total, and a shape whose copies all fit in L2 is marked ``l2_resident``.
"""

from __future__ import annotations

import argparse
import ctypes

import torch

from . import _lib

SHAPES = {"lm": (248320, 2560), "down": (2560, 9216), "q": (8192, 2560), "gate": (9216, 2560),
          "kv": (1024, 2560), "o": (2560, 4096)}

# (role, N, K): the distinct decode GEMV shapes of configs 0 and 1
DECODE_SHAPES = [
    ("MLP gate / up (config 0)", 9216, 2560),
    ("MLP down", 2560, 9216),
    ("attention q (+ output gate)", 8192, 2560),
    ("attention k / v", 1024, 2560),
    ("attention o / GDN out_proj", 2560, 4096),
    ("GDN in_proj q / k", 2048, 2560),
    ("GDN in_proj v / z", 4096, 2560),
    ("GDN in_proj a / b", 32, 2560),
]
L2_BYTES = 126 << 20


def gemv_bytes(n: int, k: int) -> int:
    """Algorithmic bytes of one GEMV: E4M3 weights, BF16 block scales, BF16 x and y."""
    return n * k + ((n + 127) // 128) * (k // 128) * 2 + 2 * k + 2 * n


def time_shapes(peak_gbs: float, shapes=DECODE_SHAPES, launches: int = 64, replays: int = 10, ref_lib=None,
                chained: bool = True) -> list:
    """Mean time per launch of each shape (see the module docstring).

    ``ref_lib``: another library exporting ``launch_gemv_v4_extern`` with the
    reference's signature (e.g. the reference's own kernels built for
    sm_100a); when given, its entry point is timed instead of ours, as
    ``abi``.  ``chained=False`` skips the PDL-chained leg."""
    P = ctypes.c_void_p
    lib = _lib.fused()
    abi_lib = ref_lib if ref_lib is not None else lib
    out = []
    for role, n, k in shapes:
        wb = n * k
        copies = max(2, min(64, -(-3 * L2_BYTES // wb)))
        nl = -(-max(launches, copies) // copies) * copies
        ws = torch.randint(0, 120, (copies, n, k), dtype=torch.uint8, device="cuda")
        s = (torch.rand((n + 127) // 128, k // 128, device="cuda") * 1e-3).to(torch.bfloat16)
        x = torch.randn(k, device="cuda").to(torch.bfloat16)
        y = torch.empty(n, dtype=torch.bfloat16, device="cuda")
        yf = torch.empty(n, dtype=torch.float32, device="cuda")

        def abi(i, st):
            abi_lib.launch_gemv_v4_extern(P(x.data_ptr()), P(ws[i].data_ptr()), P(s.data_ptr()), P(y.data_ptr()),
                                      n, k, k // 128, st)

        def chained_leg(i, st):
            _lib.check(lib.qwen_linear_partial(P(x.data_ptr()), P(ws[i].data_ptr()), P(s.data_ptr()), n, k,
                                               k // 128, P(yf.data_ptr()), st), "qwen_linear_partial")

        row = {"role": role, "shape": f"{n}x{k}", "bytes": gemv_bytes(n, k), "copies": copies,
               "cycled_mb": round(copies * wb / 2**20, 1), "l2_resident": copies * wb <= L2_BYTES}
        legs = [("abi", abi)] + ([("chained", chained_leg)] if chained else [])
        for name, fn in legs:
            st = P(torch.cuda.current_stream().cuda_stream)
            for i in range(copies):  # tensor maps built outside the capture
                fn(i, st)
            if ref_lib is None:
                _lib.check_last(f"gemv {n}x{k}")
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                cs = P(torch.cuda.current_stream().cuda_stream)
                for i in range(nl):
                    fn(i % copies, cs)
            g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(replays):
                g.replay()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1000.0 / (replays * nl)
            gbs = row["bytes"] / us / 1e3
            row[name] = {"us": round(us, 3), "gbs": round(gbs, 1), "frac": round(gbs / peak_gbs, 4)}
            del g
        out.append(row)
        del ws
        torch.cuda.empty_cache()
    err = _lib.device_error()
    if err:
        raise RuntimeError(f"device error {err} while timing GEMV shapes")
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--shapes", default="lm,down,q")
    ap.add_argument("--reps", type=int, default=2)
    ap.add_argument("--time", action="store_true", help="time every config 0/1 decode shape instead")
    args = ap.parse_args()
    P = ctypes.c_void_p
    lib = _lib.fused()
    if args.time:
        import json
        import os
        peaks = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                             "MEASURED_PEAKS.json")
        peak = float(json.load(open(peaks))["hbm_gbs"]) if os.path.exists(peaks) else 6650.0
        lib.qwen_set_pdl(1)
        for row in time_shapes(peak):
            print(json.dumps(row), flush=True)
        return
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

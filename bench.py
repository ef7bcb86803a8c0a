#!/usr/bin/env python
"""Batch-1 greedy decode throughput of the random-init Qwen3.5-4B text decoder
on B200, plus the HBM roofline of the dominant kernel.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--engine step|launch]

One step = one decode token through the whole 32-layer model.  On one GPU the
default engine runs the token as one launch of the persistent step kernel
(qwen35_b200.step); ``--engine launch`` runs the per-stage launch chain (162
kernels in one CUDA graph), which is also the tensor-parallel engine's form
for N > 1.  Timing: a 128-token seeded prompt is fed first, then W untimed
decode steps, then EXACTLY K steps bracketed by a barrier and
torch.cuda.synchronize(), timed with CUDA events on the launching stream; the
max over ranks is reported.  Every step streams ~4.3 GB of weights, far more
than the 126 MB L2, so no flush is needed between steps.

Keys beyond the base contract:
  e2e           the same K steps through the public API engine.decode() (token
                in from pinned memory, the step, next token and a sequence
                number written to pinned memory, host polls)
  roofline      the dominant kernel: the step kernel (one launch per token, all
                of the step's bytes) with the launch engine, the dominant GEMV
                kernel on the LM-head launch of config 2
  step_roofline algorithmic bytes of a whole decode step / device time per step
  stage_roofline (step kernel) per stage kind, from the kernel's own timeline
                (qwen35_b200.profile_step): bytes of the stage / its span on the
                critical path, and the span's share of the step
  lm_head_kernel the LM-head GEMV + argmax kernel of the launch engine timed alone
  gemv_shapes   (1 GPU) every config 0/1 decode GEMV shape timed alone, through the
                reference entry point and PDL-chained (qwen35_b200.profile_gemv)
  cpu_baseline  the CPU oracle port (explicit FP8->FP32 dequant + torch matmul)
                on a bounded sample of the step, scaled to tok/s, with the
                dequant and the matmul of every decode GEMV shape timed apart
  clocks        nvidia-smi samples taken during the timed region

--impl reference times the reference's path on the host CPU cores (the oracle
port; the reference has no CPU implementation of its own), rank 0 only; its
line also carries the reference's own GEMV kernel (built from its sources into
oracle/_ref) timed per decode shape on the GPU, when that build is present.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "qwen3.5-fp8-cuda_b200"))
sys.path.insert(0, REPO)

import torch  # noqa: E402

METRIC = "batch-1 decode tok/s (Qwen3.5-4B arch); FP8 GEMV achieved HBM GB/s vs peak"
UNIT = "tok/s"
PROMPT_LEN = 128


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-pdl", action="store_true", help="disable programmatic dependent launch")
    ap.add_argument("--engine", choices=["step", "launch"], default="step",
                    help="one GPU: persistent step kernel (default) or the per-stage launch chain")
    return ap.parse_args()


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_traffic(name="gemv_lm_head_config2_ncu.txt"):
    """DRAM bytes per launch from a committed ncu summary under profiles/ (the
    line ``dram_bytes_per_launch = ...``), if any."""
    path = os.path.join(REPO, "profiles", name)
    if not os.path.exists(path):
        return None
    with open(path) as f:
        for line in f:
            if line.startswith("dram_bytes_per_launch"):
                return int(float(line.split("=")[1].split()[0]))
    return None


def stage_bytes(cfg, w):
    """Algorithmic bytes per stage name of the step kernel's program (weights
    and scales of the stage's GEMVs, the GatedDeltaNet state read + write),
    summed over the step."""
    out = {}

    def add(name, *mats):
        out[name] = out.get(name, 0) + sum(tensor_bytes(m) for m in mats)

    for i, ly in enumerate(w["layers"]):
        if cfg.layer_types[i] == "full_attention":
            add("qkv", ly["q_proj"], ly["k_proj"], ly["v_proj"])
            add("o_proj", ly["o_proj"])
        else:
            add("in_proj", ly["in_proj_qkv"], ly["in_proj_z"], ly["in_proj_a"], ly["in_proj_b"])
            out["gdn"] = out.get("gdn", 0) + 2 * cfg.linear_num_value_heads * cfg.linear_key_head_dim * \
                cfg.linear_value_head_dim * 4
            add("out_proj", ly["out_proj"])
        add("gate_up", ly["gate_proj"], ly["up_proj"])
        add("down", ly["down_proj"])
    add("lm_head", w["lm_head"])
    return out


# ---------------------------------------------------------------------------
# Clock sampling during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sms.append(float(parts[0]))
                maxes.append(float(parts[1]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sms:
            return None
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
                "samples": len(sms)}


def physical_gpu_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


# ---------------------------------------------------------------------------
# Algorithmic bytes
# ---------------------------------------------------------------------------
def tensor_bytes(t):
    if isinstance(t, tuple):
        return sum(x.numel() * x.element_size() for x in t)
    return t.numel() * t.element_size()


def step_bytes(cfg, w, ctx: int, lcfg=None) -> int:
    """Bytes one decode step must move on one GPU: weights, norms, recurrent/conv
    state (read + write), KV cache read at context `ctx` plus the new row, LM
    head.  `w` and `lcfg` are the rank's shard under tensor parallelism."""
    cfg = lcfg or cfg
    total = cfg.hidden_size * 2  # embedding row
    for i, ly in enumerate(w["layers"]):
        for k, v in ly.items():
            if k == "layer_type":
                continue
            if k == "conv1d_w" or isinstance(v, tuple) or k in ("A_log", "dt_bias", "norm_w", "q_norm", "k_norm",
                                                                  "input_layernorm", "post_attention_layernorm"):
                total += tensor_bytes(v)
        if cfg.layer_types[i] == "full_attention":
            row = cfg.num_key_value_heads * cfg.head_dim * 2
            total += 2 * row * ctx + 2 * row
        else:
            total += 2 * cfg.linear_num_value_heads * cfg.linear_key_head_dim * cfg.linear_value_head_dim * 4
            total += 2 * cfg.conv_dim * cfg.linear_conv_kernel_dim * 2
    total += tensor_bytes(w["lm_head"]) + tensor_bytes(w["norm_f"])
    return total


def lm_head_bytes(cfg, w) -> int:
    wh, sh = w["lm_head"]
    return tensor_bytes((wh, sh)) + cfg.hidden_size * (2 + 4) + 16


# ---------------------------------------------------------------------------
# CPU oracle leg
# ---------------------------------------------------------------------------
UNIT_KINDS = ("linear_attention", "full_attention", "head")


def time_cpu_units(cfg, layers, head, n_units, warmup_units=1):
    """Run `n_units` decode-step units of the CPU oracle, cycling through a
    GatedDeltaNet layer, a full-attention layer and the LM head (so every
    kind of unit of a token is in every sample of three or more units);
    returns [(kind, seconds)] of the timed units."""
    from oracle import ops
    from oracle.model import OracleModel

    one_cfg = type(cfg)(**{**cfg.__dict__, "num_hidden_layers": 2, "layer_types": ["linear_attention",
                                                                                  "full_attention"]})
    wd = {"embed": torch.zeros(1, cfg.hidden_size, dtype=torch.bfloat16), "norm_f": head["norm_f"],
          "lm_head": head["lm_head"], "layers": [layers["linear_attention"], layers["full_attention"]]}
    om = OracleModel(one_cfg, wd, max_seq=64)
    hidden = (torch.randn(cfg.hidden_size, generator=torch.Generator().manual_seed(1)) * 0.5).to(torch.bfloat16)
    times = []
    for u in range(n_units + warmup_units):
        kind = UNIT_KINDS[u % 3]
        t0 = time.perf_counter()
        if kind != "head":
            li = 0 if kind == "linear_attention" else 1
            ly = wd["layers"][li]
            res = hidden
            h = ops.rmsnorm(hidden, ly["input_layernorm"])
            a = om._linear(h, ly, li) if li == 0 else om._full(h, ly, li)
            hidden = ops.mlp_post(res, a, ly["post_attention_layernorm"], *ly["gate_proj"], *ly["up_proj"],
                                  *ly["down_proj"])["output"]
            om.pos = min(om.pos + (1 if li == 1 else 0), 60)
        else:
            h = ops.rmsnorm(hidden, wd["norm_f"])
            logits = ops.gemv(h, *wd["lm_head"])
            ops.argmax_first(logits)
        dt = time.perf_counter() - t0
        if u >= warmup_units:
            times.append((kind, dt))
    return times


def cpu_sample_weights(cfg, seed=7):
    """One GDN layer, one full-attention layer and the LM head of the 4B shapes,
    generated on the CPU with the benchmark's recipe (oracle.synth)."""
    from oracle import synth
    g = synth.gen(seed)
    H, I = cfg.hidden_size, cfg.intermediate_size

    def fp8(n, k):
        w, s = synth.fp8_weight(n, k, g)
        return w, s.to(torch.bfloat16)

    def norm(n):
        return torch.randn(n, generator=g) * 0.02

    common = lambda: {"input_layernorm": norm(H), "post_attention_layernorm": norm(H),  # noqa: E731
                      "gate_proj": fp8(I, H), "up_proj": fp8(I, H), "down_proj": fp8(H, I)}
    lin = common()
    nv = cfg.linear_num_value_heads
    lin.update({"in_proj_qkv": fp8(cfg.conv_dim, H), "in_proj_a": fp8(nv, H), "in_proj_b": fp8(nv, H),
                "in_proj_z": fp8(cfg.linear_value_dim, H), "out_proj": fp8(H, cfg.linear_value_dim),
                "A_log": torch.log(torch.rand(nv, generator=g) * 15 + 1), "dt_bias": torch.ones(nv),
                "conv1d_w": (torch.randn(cfg.conv_dim, cfg.linear_conv_kernel_dim, generator=g) * 0.1).to(
                    torch.bfloat16),
                "norm_w": (1 + torch.randn(cfg.linear_value_head_dim, generator=g) * 0.02).to(torch.bfloat16)})
    full = common()
    qd = cfg.num_attention_heads * cfg.head_dim
    kvd = cfg.num_key_value_heads * cfg.head_dim
    full.update({"q_proj": fp8(2 * qd, H), "k_proj": fp8(kvd, H), "v_proj": fp8(kvd, H), "o_proj": fp8(H, qd),
                 "q_norm": norm(cfg.head_dim), "k_norm": norm(cfg.head_dim)})
    head = {"lm_head": fp8(cfg.vocab_size, H), "norm_f": norm(H)}
    return {"linear_attention": lin, "full_attention": full}, head


def cpu_tok_per_s(cfg, times):
    """Scale per-unit medians to one full decode step (24 GDN + 8 full layers + head)."""
    per = {k: [dt for kind, dt in times if kind == k] for k in UNIT_KINDS}
    t_lin = statistics.median(per["linear_attention"]) if per["linear_attention"] else 0.0
    t_full = statistics.median(per["full_attention"]) if per["full_attention"] else t_lin
    t_head = statistics.median(per["head"]) if per["head"] else 0.0
    n_lin = cfg.layer_types.count("linear_attention")
    n_full = cfg.num_hidden_layers - n_lin
    step = n_lin * t_lin + n_full * t_full + t_head
    return 1.0 / step, step


def decode_gemv_shapes(cfg):
    """[(N, K, launches per token)] of every linear weight of one decode step."""
    H, I = cfg.hidden_size, cfg.intermediate_size
    n_lin = cfg.layer_types.count("linear_attention")
    n_full = cfg.num_hidden_layers - n_lin
    qd = cfg.num_attention_heads * cfg.head_dim
    kvd = cfg.num_key_value_heads * cfg.head_dim
    nv = cfg.linear_num_value_heads
    return [(I, H, 2 * cfg.num_hidden_layers), (H, I, cfg.num_hidden_layers),
            (2 * qd, H, n_full), (kvd, H, 2 * n_full), (H, qd, n_full),
            (cfg.conv_dim, H, n_lin), (cfg.linear_value_dim, H, n_lin), (nv, H, 2 * n_lin),
            (H, cfg.linear_value_dim, n_lin), (cfg.vocab_size, H, 1)]


def cpu_gemv_split(cfg, runs=10):
    """The reference path's two host costs per token, timed apart: the
    explicit FP8 -> FP32 block dequantisation (main.py:497-501) and the FP32
    matmul, each the median of `runs` runs per decode GEMV shape, summed over
    the shapes' launches per token."""
    from oracle import ops, synth
    g = synth.gen(11)
    dq_total = mm_total = 0.0
    rows = []
    for n, k, count in decode_gemv_shapes(cfg):
        w, s32 = synth.fp8_weight(n, k, g)
        s = s32.to(torch.bfloat16)
        x = synth.bf16_vector(k, g).float()
        t_dq, t_mm = [], []
        for _ in range(runs):
            t0 = time.perf_counter()
            wd = ops.dequant(w, s)
            t1 = time.perf_counter()
            (wd @ x).to(torch.bfloat16)
            t2 = time.perf_counter()
            t_dq.append(t1 - t0)
            t_mm.append(t2 - t1)
        dq, mm = statistics.median(t_dq), statistics.median(t_mm)
        dq_total += count * dq
        mm_total += count * mm
        rows.append({"shape": f"{n}x{k}", "per_token": count, "dequant_ms": round(dq * 1e3, 3),
                     "matmul_ms": round(mm * 1e3, 3)})
        del w, wd
    return {"dequant_s_per_token": round(dq_total, 4), "matmul_s_per_token": round(mm_total, 4),
            "sum_s_per_token": round(dq_total + mm_total, 4), "runs_per_shape": runs,
            "statistic": "median", "shapes": rows}


def run_cpu_baseline(cfg, n_units=33):
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    layers, head = cpu_sample_weights(cfg)
    times = time_cpu_units(cfg, layers, head, n_units)
    tps, step_s = cpu_tok_per_s(cfg, times)
    out = {"value": round(tps, 6), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
           "sample": f"{n_units} units of one decode step cycling GDN layer / full-attention layer / LM head at "
                     f"4B shapes (explicit FP8->FP32 dequant + torch matmul), median per unit kind, scaled to "
                     f"24 GDN + 8 full layers + head = {step_s:.3f} s/token"}
    try:
        out["gemv_split"] = cpu_gemv_split(cfg)
    except Exception as exc:  # reported, never allowed to drop the baseline
        out["gemv_split"] = {"error": repr(exc)[:200]}
    return out


# ---------------------------------------------------------------------------
# Reference arm: the reference's path on the host CPU (oracle port)
# ---------------------------------------------------------------------------
def ref_gpu_gemv_shapes(peak):
    """The reference's own GEMV kernel (launch_gemv_v4_extern of
    fused_kernels.cu:1328-1336, built unmodified for sm_100a into oracle/_ref)
    timed per config 0/1 decode shape on this GPU, by the same method as the
    gemv_shapes leg of our arm; None when that build or a GPU is absent."""
    path = os.path.join(REPO, "oracle", "_ref", "libref_fused.so")
    if not (os.path.exists(path) and torch.cuda.is_available()):
        return None
    import ctypes
    from qwen35_b200.profile_gemv import time_shapes
    ref = ctypes.CDLL(path)
    ref.launch_gemv_v4_extern.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 3 + [ctypes.c_void_p]
    ref.launch_gemv_v4_extern.restype = None
    return time_shapes(peak, ref_lib=ref, chained=False)


def ref_gpu_engine(steps=30, warmup=3):
    """The reference's default decode step re-driven on this GPU through its
    own kernels (oracle.ref_engine: main.py:1509-1604 with fused_kernels.cu
    built unmodified for sm_100a), at the 4B shapes from position 128; and its
    delta-rule kernel alone (launch_delta_rule_decode, 32 heads).  None when
    the build or a GPU is absent."""
    path = os.path.join(REPO, "oracle", "_ref", "libref_fused.so")
    if not (os.path.exists(path) and torch.cuda.is_available()):
        return None
    import ctypes
    from oracle.ref_engine import ReferenceKernelEngine
    from qwen35_b200.config import qwen35_4b
    from qwen35_b200.weights import random_weights
    cfg = qwen35_4b()
    w = random_weights(cfg, seed=0, device="cuda")
    eng = ReferenceKernelEngine(cfg, w, max_seq=PROMPT_LEN + steps + warmup + 8)
    eng.pos = PROMPT_LEN
    tok = 7
    for _ in range(warmup):
        _, tok = eng.step(tok)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        _, tok = eng.step(tok)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    out = {"what": "reference decode step (its kernels from oracle/_ref, its torch ops restated), 4B shapes, "
                   f"positions {PROMPT_LEN}-{PROMPT_LEN + steps}", "ms_per_step": round(ms, 3),
           "tok_per_s": round(1000.0 / ms, 2)}
    H, D = cfg.linear_num_value_heads, cfg.linear_value_head_dim
    g = torch.Generator(device="cuda").manual_seed(1)
    q, k = (torch.randn(H, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(2))
    v = torch.randn(H, D, generator=g, device="cuda").to(torch.bfloat16)
    gg = -torch.rand(H, generator=g, device="cuda")
    beta = torch.rand(H, generator=g, device="cuda").to(torch.bfloat16)
    state = torch.randn(H, D, D, generator=g, device="cuda") * 0.1
    o = torch.empty(H, D, dtype=torch.bfloat16, device="cuda")
    P = ctypes.c_void_p
    args = [P(t.data_ptr()) for t in (q, k, v, gg, beta, state, o)]
    for _ in range(5):
        eng.lib.launch_delta_rule_decode(*args, H, D, P(0))
    torch.cuda.synchronize()
    e0.record()
    for _ in range(100):
        eng.lib.launch_delta_rule_decode(*args, H, D, P(0))
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 10.0
    out["delta_rule_decode"] = {"us_per_launch": round(us, 2), "heads": H,
                                "gbs_state": round(2 * H * D * D * 4 / us / 1e3, 1)}
    return out


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from qwen35_b200.config import qwen35_4b
    cfg = qwen35_4b()
    torch.set_num_threads(os.cpu_count() or 1)
    layers, head = cpu_sample_weights(cfg)
    # each step is one unit of a decode token, cycling GDN layer / full-attention
    # layer / LM head, so every kind is timed whatever K is (K >= 3)
    times = time_cpu_units(cfg, layers, head, max(3, args.steps), warmup_units=args.warmup)
    tps, step_s = cpu_tok_per_s(cfg, times)
    line = {
        "metric": METRIC, "value": round(tps, 6), "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * step_s, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_block(args),
        "cpu_baseline": {"value": round(tps, 6), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"{len(times)} timed units cycling GDN layer / full-attention layer / LM head "
                                   f"(4B shapes), explicit FP8->FP32 dequant + torch matmul; medians per kind "
                                   f"scaled to one token (24 GDN + 8 full + head) = {step_s:.3f} s"},
        "e2e": {"value": round(tps, 6), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    try:
        peak, _ = load_peaks()
        rows = ref_gpu_gemv_shapes(peak)
        if rows is not None:
            line["ref_gpu_gemv_shapes"] = {
                "kernel": "reference gemv_v4_kernel via launch_gemv_v4_extern (oracle/_ref, sm_100a build of "
                          "fused_kernels.cu)", "unit": "us per launch; GB/s of algorithmic bytes",
                "rows": rows}
    except Exception as exc:  # context only, never allowed to drop the line
        line["ref_gpu_gemv_shapes"] = {"error": repr(exc)[:200]}
    try:
        r = ref_gpu_engine()
        if r is not None:
            line["ref_gpu_engine"] = r
    except Exception as exc:  # context only, never allowed to drop the line
        line["ref_gpu_engine"] = {"error": repr(exc)[:200]}
    print(json.dumps(line), flush=True)


def config_block(args):
    return {"workload": "config3: random-init Qwen3.5-4B text decoder, 128-token seeded prompt, batch-1 greedy "
                        "decode (E4M3 128x128 block-scaled linear weights incl. LM head)",
            "model": "Qwen3.5-4B (random init)", "global_batch": 1, "prompt_len": PROMPT_LEN,
            "decode_steps": args.steps, "parallelism": f"tp{args.gpus}" if args.gpus > 1 else "single",
            **({"tp_exchange": "step kernel, Megatron-style split: column-parallel in_proj / qkv / gate-up / LM "
                               "head, row-parallel out_proj / o_proj / down whose FP32 K-slice rows every CTA "
                               "stores on every rank over NVLink (CUDA IPC peer memory, no library collective); "
                               "two cross-GPU hand-offs per layer"}
               if args.gpus > 1 else {}),
            "l2": "no flush: each step streams ~4.3 GB of weights (> 126 MB L2)"}


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    from qwen35_b200 import _lib
    from qwen35_b200.config import qwen35_4b
    from qwen35_b200.engine import Qwen35DecodeEngine
    from qwen35_b200.step import Qwen35StepEngine
    from qwen35_b200.tp import Qwen35TPDecodeEngine
    from qwen35_b200.weights import random_weights

    if args.no_pdl:
        _lib.fused().qwen_set_pdl(0)
    cfg = qwen35_4b()
    w = random_weights(cfg, seed=args.seed, device="cuda")
    max_seq = PROMPT_LEN + args.warmup + 2 * args.steps + 16
    if world > 1 and args.engine == "step":
        # tensor parallel on the step kernel: one decode stream over all ranks,
        # every stage sharded, outputs stored on every rank over NVLink
        from qwen35_b200.step_tp import Qwen35StepTPEngine
        eng = Qwen35StepTPEngine(cfg, w, rank, world, max_seq=max_seq)
    elif world > 1:
        # tensor parallel on the per-launch engine (every rank holds the same
        # full random weights and keeps its shard)
        eng = Qwen35TPDecodeEngine(cfg, w, rank, world, max_seq=max_seq)
        del w
        torch.cuda.empty_cache()
    elif args.engine == "step":
        eng = Qwen35StepEngine(cfg, w, max_seq=max_seq)
    else:
        eng = Qwen35DecodeEngine(cfg, w, max_seq=max_seq)
    step_engine = isinstance(eng, Qwen35StepEngine)
    eng.capture()
    g = torch.Generator().manual_seed(1000 + args.seed)
    prompt = torch.randint(0, cfg.vocab_size, (PROMPT_LEN,), generator=g).tolist()
    for t in prompt:
        eng.decode(t)
    for _ in range(args.warmup):
        eng.step()
    torch.cuda.synchronize()
    sampler = ClockSampler(physical_gpu_index(local))
    sampler.start()
    time.sleep(0.2)
    ctx0 = eng.position()

    # device-resident greedy loop: K graph replays
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        eng.step()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    dev_ms = max_over_ranks(e0.elapsed_time(e1))

    # end to end through the public API: token H2D, replay, token D2H, sync
    tok = int(eng.token.item())
    barrier()
    torch.cuda.synchronize()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record()
    for _ in range(args.steps):
        tok = eng.decode(tok)
    e3.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e2.elapsed_time(e3))
    clocks = sampler.stop()
    assert _lib.device_error() == 0, "device error word set (bounded wait timed out)"

    # the launch engine's LM-head streaming GEMV + argmax kernel alone (config 2
    # launch; this rank's vocabulary shard under tensor parallelism)
    wh, sh = eng.w["lm_head"]
    row_offset = eng.w.get("lm_row_offset", 0)
    ws = torch.zeros(2, dtype=torch.int64, device="cuda")
    key = torch.zeros(1, dtype=torch.int64, device="cuda")
    tokb = torch.zeros(1, dtype=torch.int64, device="cuda")
    import ctypes
    P = ctypes.c_void_p
    lib = _lib.fused()
    stream = P(torch.cuda.current_stream().cuda_stream)

    def head_launch():
        _lib.check(lib.launch_lm_head_argmax(P(eng.hidden.data_ptr()), P(eng.w["norm_f"].data_ptr()), 1e-6,
                                             P(wh.data_ptr()), P(sh.data_ptr()), wh.shape[0], wh.shape[1],
                                             wh.shape[1] // 128, row_offset, P(ws.data_ptr()), P(key.data_ptr()),
                                             P(tokb.data_ptr()), P(0), P(0), stream), "lm head")

    for _ in range(3):
        head_launch()
    reps = 20
    torch.cuda.synchronize()
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0.record()
    for _ in range(reps):
        head_launch()
    h1.record()
    torch.cuda.synchronize()
    head_s = h0.elapsed_time(h1) / 1000.0 / reps
    peak, peak_kind = load_peaks()
    hb = wh.numel() + sh.numel() * sh.element_size() + 2 * cfg.hidden_size + 8
    head_gbs = hb / head_s / 1e9
    sbytes = step_bytes(cfg, eng.w, ctx0 + args.steps // 2, eng.cfg)
    step_s = dev_ms / 1000.0 / args.steps
    step_gbs = sbytes / step_s / 1e9
    head_kernel = {"kernel": "gemv_tcw_kernel<bf16,false> (tcgen05 N=256 + TMA) on the LM head "
                             "(248320x2560 E4M3, config 2)", "achieved": round(head_gbs, 1), "unit": "GB/s",
                   "frac": round(head_gbs / peak, 4), "bytes_per_launch": hb, "us_per_launch": round(head_s * 1e6, 2),
                   "traffic": load_traffic()}
    head_stage = None
    if step_engine:
        # config 2 on the step kernel, E4M3 and BF16 heads (one-stage programs)
        try:
            from qwen35_b200.profile_step import head_stage_rate
            head_stage = {"unit": "GB/s of algorithmic bytes (weights, scales, x); frac of the measured peak",
                          "shape": "248320x2560, x BF16, fused greedy argmax, one step-kernel launch per GEMV"}
            for name, fp8 in (("e4m3", True), ("bf16", False)):
                r = head_stage_rate(fp8=fp8)
                r["frac"] = round(r["gbs"] / peak, 4)
                head_stage[name] = r
        except Exception as exc:  # reported, never allowed to drop the line
            head_stage = {"error": repr(exc)[:200]}
    if step_engine:
        # the dominant (only) kernel of a step: the persistent step kernel; one
        # launch per step, so its launch time is the device time per step.
        # Tensor parallel: each rank's launch streams its 1/world share.
        rank_bytes = sbytes // world
        rank_gbs = rank_bytes / step_s / 1e9
        traffic = load_traffic("step_kernel_config3_ncu.txt")
        roofline = {"bound": "hbm", "achieved": round(rank_gbs, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(rank_gbs / peak, 4), "traffic": traffic if world == 1 else None,
                    "kernel": "step_kernel (persistent, one cooperative launch per token: every GEMV, GatedDeltaNet, "
                              "attention and LM-head stage" + (f"; one per GPU, ~1/{world} of every stage)"
                                                               if world > 1 else ")"),
                    "bytes_per_launch": rank_bytes, "us_per_launch": round(step_s * 1e6, 2), "peak_kind": peak_kind}
    else:
        roofline = {"bound": "hbm", **{k: v for k, v in head_kernel.items() if k != "kernel"}, "peak": peak,
                    "peak_kind": peak_kind, "kernel": head_kernel["kernel"]}

    line = {
        "metric": METRIC,
        "value": round(args.steps / (dev_ms / 1000.0), 3),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dev_ms / args.steps, 5),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "e4m3xbf16->f32",
        "data": "synthetic (seeded random-init weights and prompt ids)",
        "config": {**config_block(args), "engine": "step" if step_engine else "launch"},
        "e2e": {"value": round(args.steps / (e2e_ms / 1000.0), 3), "unit": UNIT,
                "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8},
        "gpu_launches": eng.kernels_per_step * args.steps,
        "roofline": roofline,
        "step_roofline": {"bytes_per_step": sbytes, "achieved": round(step_gbs, 1),
                          "frac": round(step_gbs / peak, 4), "unit": "GB/s"},
        "lm_head_kernel": head_kernel,
        "lm_head_step_stage": head_stage,
        "clocks": clocks,
        "pdl": not args.no_pdl,
    }
    if step_engine:
        try:
            from qwen35_b200 import profile_step
            rows = profile_step.summarize(cfg, profile_step.timeline(eng))
            sb = stage_bytes(cfg, eng.w)
            agg = {}
            for r in rows:
                a = agg.setdefault(r["name"], {"stages": 0, "span_us": 0.0})
                a["stages"] += 1
                a["span_us"] += r["span"] / 1000.0
            total = sum(a["span_us"] for a in agg.values())
            for name, a in agg.items():
                b = sb.get(name, 0)
                a["bytes"] = b
                a["gbs"] = round(b / (a["span_us"] * 1e3), 1) if a["span_us"] else None
                a["frac"] = round(a["gbs"] / peak, 4) if a["gbs"] else None
                a["share"] = round(a["span_us"] / total, 4)
                a["span_us"] = round(a["span_us"], 1)
            line["stage_roofline"] = {"unit": "GB/s of the stage's algorithmic bytes over its span on the step's "
                                              "critical path (one timed step)", "stages": agg}
        except Exception as exc:  # reported, never allowed to drop the line
            line["stage_roofline"] = {"error": repr(exc)[:200]}
    if world == 1:
        # every config 0/1 decode GEMV shape alone (after the timed region)
        from qwen35_b200.profile_gemv import time_shapes
        try:
            rows = time_shapes(peak)
        except Exception as exc:  # reported, never allowed to drop the line
            rows = {"error": repr(exc)[:200]}
        line["gemv_shapes"] = {
            "unit": "us per launch; GB/s of algorithmic bytes; frac of the measured peak",
            "method": "CUDA graph of back-to-back launches over rotating weight copies; abi = "
                      "launch_gemv_v4_extern (no PDL), chained = qwen_linear_partial (PDL)",
            "rows": rows}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = run_cpu_baseline(cfg)
        except Exception as exc:  # the baseline is reported, never required
            line["cpu_baseline"] = {"value": None, "error": repr(exc)[:200]}
    eng.graph = None
    eng.graph_io = None
    if world > 1:
        eng.close()
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

"""Stage timeline of the persistent decode-step kernel.

    python -m qwen35_b200.profile_step [--layers N] [--context N] [--steps N] [--per-stage]

Builds the random-init Qwen3.5-4B step engine (optionally with fewer layers),
runs warm-up steps, then one step with the kernel's timeline on
(``qwen_step_set_timeline``): per stage and CTA the consumers' wait for the
previous stage begins / ends, their work ends, and the producer's first / last
issue of the stage's items, all from ``%globaltimer``.  Prints, per stage
name, where the step's time goes:

* ``span``: from the previous stage's last CTA finishing to this stage's last
  CTA finishing (the stage's share of the step's critical path);
* ``sync``: from the previous stage's last CTA finishing to the median CTA
  starting this stage (the cost of the grid-wide dependency);
* ``work``: median and max over CTAs of the stage's own work;
* ``lead``: how far ahead of the stage's start the median producer had
  issued the stage's last item (negative: the stream was behind);
* ``pblk`` / ``cblk``: median ns the producer was blocked on a full ring while
  issuing the stage / consumer warp 0 was blocked on copies not yet landed
  (a producer blocked means the consumers set the pace; consumers blocked
  means the stream does);
* ``pro``: median time from the stage's start to its x prologue being done;
* ``chunk``: median time from the prologue's end to the last batch's chunk
  math being done; ``wcomp``: consumer warp 0's SM clock cycles (thousands)
  inside the chunk math.  For GatedDeltaNet stages ``pro`` is the time to the
  head's inputs having arrived and ``chunk`` the state update after that; for
  attention stages ``pro`` is the q / k / v preparation, ``chunk`` the
  positions up to the published partials, ``wcomp`` the combine (us).

Also prints the step time measured with CUDA events over ``--steps`` steps.
"""

from __future__ import annotations

import argparse
import ctypes
import statistics

import torch

KINDS = {0: "gemv", 1: "gdn", 2: "attn"}
NF = 10  # timeline words per (stage, CTA)


def stage_names(cfg):
    """Short names of the engine's stages, in program order."""
    names = []
    for lt in cfg.layer_types:
        names += ["qkv", "attn", "o_proj"] if lt == "full_attention" else ["in_proj", "gdn", "out_proj"]
        names += ["gate_up", "down"]
    names.append("lm_head")
    return names


def kinds_of(eng):
    return [KINDS[st.kind] for st in eng.stages]


def timeline(eng):
    """One step with the timeline on: [stages, grid, 10] int64 (stamps in ns from the earliest one)."""
    ns, grid = len(eng.stages), eng.grid
    buf = torch.zeros(ns * grid * NF, dtype=torch.int32, device=eng.device)
    eng.lib.qwen_step_set_timeline(eng.prog, ctypes.c_void_p(buf.data_ptr()))
    eng.step_eager()  # a captured graph holds the launch parameters it was captured with
    torch.cuda.synchronize(eng.device)
    eng.lib.qwen_step_set_timeline(eng.prog, ctypes.c_void_p(0))
    t = (buf.cpu().to(torch.int64) & 0xFFFFFFFF).view(ns, grid, NF)
    base = int(t[0, :, 0].min())
    t[:, :, :5] = (t[:, :, :5] - base) % (1 << 32)
    kinds = kinds_of(eng)
    for f in (7, 8, 9):
        nz = t[:, :, f] != 0
        if f == 9:  # warp-0 cycles for GEMV stages, a stamp for attention stages
            nz &= torch.tensor([k == "attn" for k in kinds]).view(-1, 1)
        t[:, :, f] = torch.where(nz, (t[:, :, f] - base) % (1 << 32), t[:, :, f])
    return t


def _med_since(stamp, since):
    """Median over the CTAs that recorded `stamp` (non-zero) of stamp - since."""
    m = (stamp != 0) & (since != 0)
    if not bool(m.any()):
        return 0
    return max(0, int((stamp[m] - since[m]).median()))


def summarize(cfg, t, kinds=None):
    names = stage_names(cfg)
    rows = []
    prev_end = int(t[0, :, 0].min())
    for s in range(t.shape[0]):
        start, end, p1 = t[s, :, 1], t[s, :, 2], t[s, :, 4]
        last_end = int(end.max())
        work = (end - start).tolist()
        rows.append(dict(stage=s, name=names[s] if s < len(names) else str(s), span=last_end - prev_end,
                         sync=int(start.median()) - prev_end, work_med=statistics.median(work), work_max=max(work),
                         lead=int(start.median()) - int(p1.median()),
                         pblk=int(t[s, :, 5].median()), cblk=int(t[s, :, 6].median()),
                         pro=_med_since(t[s, :, 7], start),
                         chunks=_med_since(t[s, :, 8], t[s, :, 7]),
                         wcomp=int(t[s, :, 9].median()) if kinds is None or kinds[s] == "gemv" else
                         _med_since(t[s, :, 9], t[s, :, 8])))
        prev_end = last_end
    return rows


def report(cfg, t, per_stage=False, out=print, kinds=None):
    rows = summarize(cfg, t, kinds)
    total = int(t[:, :, 2].max()) - int(t[0, :, 0].min())
    out(f"timeline step: {total / 1000:.1f} us")
    agg = {}
    for r in rows:
        a = agg.setdefault(r["name"], dict(n=0, span=0, sync=0, work_med=0, work_max=0, lead=0, pblk=0, cblk=0, pro=0, chunks=0,
                                             wcomp=0))
        a["n"] += 1
        for k in ("span", "sync", "work_med", "work_max", "lead", "pblk", "cblk", "pro", "chunks", "wcomp"):
            a[k] += r[k]
    out(f"{'stage':10s} {'n':>4s} {'span us':>9s} {'share':>6s} {'sync us':>8s} {'work med':>9s} {'work max':>9s} "
        f"{'lead us':>8s} {'pblk us':>8s} {'cblk us':>8s} {'pro us':>7s} {'chunk us':>8s} {'wcomp kcyc':>10s}"
        "  (per-stage means)")
    for name, a in agg.items():
        n = a["n"]
        out(f"{name:10s} {n:4d} {a['span'] / n / 1000:9.2f} {a['span'] / total:6.1%} {a['sync'] / n / 1000:8.2f} "
            f"{a['work_med'] / n / 1000:9.2f} {a['work_max'] / n / 1000:9.2f} {a['lead'] / n / 1000:8.2f} "
            f"{a['pblk'] / n / 1000:8.2f} {a['cblk'] / n / 1000:8.2f} {a['pro'] / n / 1000:7.2f} "
            f"{a['chunks'] / n / 1000:8.2f} {a['wcomp'] / n / 1000:10.2f}")
    if per_stage:
        for r in rows:
            out(str(r))
    return rows


def head_stage_rate(fp8: bool = True, reps: int = 20, seed: int = 12):
    """Config 2 on the step kernel: a one-stage program (x given, fused argmax)
    over the 248320 x 2560 LM head, E4M3 with 128 x 128 block scales or BF16
    (N(0, 0.02)).  Returns {us_per_launch, bytes_per_launch, gbs}: algorithmic
    bytes (weights, scales, x) over the CUDA-event time of `reps` launches."""
    import ctypes as C
    from . import _lib
    from .step import EPI_ARGMAX, GEMV, PRO_PLAIN, StepSeg, StepStage, create_program, pack_linear, pack_linear_bf16
    V, H = 248320, 2560
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(H, generator=g, device="cuda").to(torch.bfloat16)
    if fp8:
        from .weights import _fp8
        w, sc = _fp8(V, H, g, "cuda")
        packed = pack_linear(w, sc)
        nbytes = w.numel() + sc.numel() * sc.element_size() + 2 * H
        del w
    else:
        w = (torch.randn(V, H, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        packed = pack_linear_bf16(w)
        nbytes = w.numel() * 2 + 2 * H
        del w
    am_ws = torch.zeros(2, dtype=torch.int64, device="cuda")
    key = torch.zeros(1, dtype=torch.int64, device="cuda")
    tok = torch.zeros(1, dtype=torch.int64, device="cuda")
    seg = StepSeg()
    seg.w, seg.n, seg.epi = packed.data_ptr(), V, EPI_ARGMAX
    st = StepStage()
    st.kind, st.K, st.pro, st.nseg, st.wbf16 = GEMV, H, PRO_PLAIN, 1, 0 if fp8 else 1
    st.x = x.data_ptr()
    st.seg[0] = seg
    st.am_ws, st.am_key_out, st.am_token_out = am_ws.data_ptr(), key.data_ptr(), tok.data_ptr()
    prog = create_program([st])
    lib = _lib.fused()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(3):
        _lib.check(lib.qwen_step_launch(prog, stream), "qwen_step_launch")
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        _lib.check(lib.qwen_step_launch(prog, stream), "qwen_step_launch")
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / reps
    lib.qwen_step_destroy(prog)
    return {"us_per_launch": round(us, 2), "bytes_per_launch": nbytes, "gbs": round(nbytes / us / 1e3, 1)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--context", type=int, default=128)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--per-stage", action="store_true")
    args = ap.parse_args()
    from .config import qwen35_4b
    from .step import Qwen35StepEngine
    from .weights import random_weights
    cfg = qwen35_4b(num_hidden_layers=args.layers)
    w = random_weights(cfg, seed=0, device="cuda")
    eng = Qwen35StepEngine(cfg, w, max_seq=max(512, args.context + args.steps + 16))
    eng.pos.fill_(args.context)
    eng.token.fill_(7)
    for _ in range(3):
        eng.step()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        eng.step()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / args.steps
    print(f"step: {ms * 1000:.1f} us ({1000 / ms:.1f} tok/s), {len(eng.stages)} stages, grid {eng.grid}")
    report(cfg, timeline(eng), args.per_stage, kinds=kinds_of(eng))


if __name__ == "__main__":
    main()
